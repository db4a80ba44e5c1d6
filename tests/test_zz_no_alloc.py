"""smelb_frozen_experts_fwd_noalloc (include/smelb.h) against smelb_frozen_experts_fwd on the same inputs.

The no-allocation variant serves callers that cannot allocate device memory per call (a host binding of the C ABI
alone has no caching allocator, and a cudaMalloc / cudaFree pair per call would synchronise the device every time).
It keeps its intermediate in a file-scope device array shared by all calls, so this file is named to be collected
last and checks two calls in a row, each against the allocating entry point, with the tolerance the other expert
tests use (max relative error 2e-2, cosine 0.9999); the status head of the shared array must read 0 after them. A
fresh process checks that a call allocates nothing: free device memory is unchanged across it and exactly its two
GEMM launches run."""
import os
import subprocess
import sys

import pytest
import torch

import oracle.moe_oracle as O

pytestmark = pytest.mark.gpu

REL, COS = 2e-2, 0.9999
SCRATCH_BYTES = 33554432  # SMELB_NOALLOC_SCRATCH_BYTES


def _case(dev, seed, H, I, counts):
    import smelb
    g = torch.Generator(device=dev).manual_seed(seed)
    E = len(counts)
    gu = torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.05
    dn = torch.randn(E, H, I, generator=g, device=dev) * 0.05
    bank = smelb.Int4Experts.from_bf16(gu.bfloat16(), dn.bfloat16())
    xs = torch.randn(sum(counts), H, generator=g, device=dev).bfloat16()
    return bank.kernel_operands(), xs, torch.tensor(counts, dtype=torch.int32, device=dev)


def _run(name, ops, xs, counts_t, I, act, with_a_buf):
    from smelb import _lib
    dev = xs.device
    R, H = xs.shape
    h = torch.full((R, 2 * I), float("nan"), dtype=torch.bfloat16, device=dev)
    out = torch.full((R, H), float("nan"), dtype=torch.bfloat16, device=dev)
    args = [_lib.ptr(xs), R, H, I, _lib.ptr(counts_t), counts_t.numel(), _lib.ptr(ops["gu_q"]), _lib.ptr(ops["gu_sz"]),
            _lib.ptr(ops["dn_q"]), _lib.ptr(ops["dn_sz"]), _lib.ACT[act], _lib.ptr(h)]
    if with_a_buf:
        args.append(_lib.ptr(torch.empty(R, I, dtype=torch.bfloat16, device=dev)))
    args += [_lib.ptr(out), _lib.stream_ptr(dev)]
    _lib.call(name, *args)
    return out, h


def _close(a, b, what):
    e, c = O.rel_err(a.float().cpu(), b.float().cpu()), O.cosine(a.float().cpu(), b.float().cpu())
    assert e <= REL and c >= COS, f"{what}: rel err {e:.3e}, cosine {c:.6f}"


def test_noalloc_matches_allocating_entry_point_two_calls():
    import smelb
    dev = torch.device("cuda:0")
    cases = [  # two calls in a row with different shapes, routing and activations through the shared array
        dict(seed=11, H=512, I=256, counts=[0, 5, 300, 17, 64, 1, 0, 130], act="silu"),
        dict(seed=12, H=704, I=192, counts=[90, 0, 0, 33, 250, 7, 64, 2, 1, 40], act="gelu_tanh"),
    ]
    prepared = [(_case(dev, c["seed"], c["H"], c["I"], c["counts"]), c) for c in cases]
    got = []
    for (ops, xs, counts_t), c in prepared:
        got.append(_run("smelb_frozen_experts_fwd_noalloc", ops, xs, counts_t, c["I"], c["act"], False))
    for ((ops, xs, counts_t), c), (out, h) in zip(prepared, got):
        ref_out, ref_h = _run("smelb_frozen_experts_fwd", ops, xs, counts_t, c["I"], c["act"], True)
        assert torch.isfinite(out.float()).all() and torch.isfinite(h.float()).all()
        _close(out, ref_out, f"noalloc out (seed {c['seed']})")
        _close(h, ref_h, f"noalloc h (seed {c['seed']})")
    assert smelb.read_status() == 0
    assert _noalloc_status(dev) == (0, 0, 0, 0)


def _noalloc_status(dev, reset=True):
    import ctypes
    from smelb import _lib
    w = (ctypes.c_int32 * 4)()
    _lib.call("smelb_frozen_experts_fwd_noalloc_status", dev.index or 0, w, 1 if reset else 0)
    return tuple(w)


_FRESH = r"""
import sys, torch
sys.path[:0] = [{root!r}, {pkg!r}]
from smelb import _lib
import test_zz_no_alloc as T
dev = torch.device("cuda:0")
ops, xs, counts_t = T._case(dev, 21, 512, 256, [7, 0, 190, 64, 3])
R, H, I = xs.shape[0], 512, 256
out = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
args = [_lib.ptr(xs), R, H, I, _lib.ptr(counts_t), counts_t.numel(), _lib.ptr(ops["gu_q"]), _lib.ptr(ops["gu_sz"]),
        _lib.ptr(ops["dn_q"]), _lib.ptr(ops["dn_sz"]), _lib.ACT["silu"], None, _lib.ptr(out), _lib.stream_ptr(dev)]
_lib.call("smelb_frozen_experts_fwd_noalloc", *args)   # warm-up: module load, symbol address
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info(0)[0]
n0 = _lib.launch_count()
_lib.call("smelb_frozen_experts_fwd_noalloc", *args)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info(0)[0]
n1 = _lib.launch_count()
print("FREE", free0, free1, "LAUNCHES", n1 - n0)
assert free1 == free0, (free0, free1)
assert n1 - n0 == 2, n1 - n0
assert T._noalloc_status(dev) == (0, 0, 0, 0)
print("FRESH_OK")
"""


def test_noalloc_allocates_nothing_in_a_fresh_process():
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    code = _FRESH.format(root=root, pkg=os.path.join(root, "smel-ft_b200"))
    r = subprocess.run([sys.executable, "-c", code], cwd=here, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, PYTHONPATH=here))
    assert r.returncode == 0 and "FRESH_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_noalloc_rejects_rows_beyond_scratch():
    import smelb
    from smelb import _lib
    dev = torch.device("cuda:0")
    H, I = 256, 128
    (ops, xs, counts_t) = _case(dev, 13, H, I, [3, 5])
    out = torch.empty(8, H, dtype=torch.bfloat16, device=dev)
    too_many = SCRATCH_BYTES // (2 * I) + 1
    with pytest.raises(smelb.SmelbError, match="exceeds"):
        _lib.call("smelb_frozen_experts_fwd_noalloc", _lib.ptr(xs), too_many, H, I, _lib.ptr(counts_t), 2,
                  _lib.ptr(ops["gu_q"]), _lib.ptr(ops["gu_sz"]), _lib.ptr(ops["dn_q"]), _lib.ptr(ops["dn_sz"]),
                  _lib.ACT["silu"], None, _lib.ptr(out), _lib.stream_ptr(dev))
