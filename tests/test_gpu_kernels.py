"""GPU parity of the bit-exact pieces (int4 unpack/dequant, routing given logits, dispatch) against the CPU oracle,
through the C ABI."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    return torch.device("cuda:0")


def _status_ok():
    import smelb
    assert smelb.read_status() == 0


def test_dequant_bit_exact_vs_oracle(dev, golden):
    import smelb
    d = golden("quant.pt")
    q, s, z = d["q"].to(dev), d["scale"].to(dev), d["zero"].to(dev)
    f32 = smelb.dequant_int4(q, s, z, torch.float32).cpu()
    assert torch.equal(f32, O.dequant_int4(d["q"], d["scale"], d["zero"], torch.float32))
    assert torch.equal(f32, d["deq_f32"])  # the reference's own fp32 dequant
    b16 = smelb.dequant_int4(q, s, z, torch.bfloat16).cpu()
    ref = O.dequant_int4(d["q"], d["scale"], d["zero"], torch.float32).to(torch.bfloat16)
    assert torch.equal(b16.view(torch.int16), ref.view(torch.int16))
    _status_ok()


def test_dequant_any_expert_count_and_group(dev):
    import smelb
    g = torch.Generator(device=dev).manual_seed(3)
    w = torch.randn(9, 64, 256, generator=g, device=dev) * 0.05
    for group in (64, 32, 128):
        pk = smelb.quantize_int4(w, group)
        for e1 in (1, 3, 9):
            a = smelb.dequant_int4(pk["q"][:e1], pk["scale"][:e1], pk["zero"][:e1], torch.float32).cpu()
            b = O.dequant_int4(pk["q"][:e1].cpu(), pk["scale"][:e1].cpu(), pk["zero"][:e1].cpu())
            assert torch.equal(a, b)


def test_quantize_matches_reference(dev, golden):
    """GPU quantizer vs the reference's CPU output: codes and (scale, zero) equal except where the clip search's
    squared errors tie to within fp32 rounding (summation order differs between CPU and GPU)."""
    import smelb
    d = golden("quant.pt")
    pk = smelb.quantize_int4(d["w"].to(dev), 64)
    same_s = (pk["scale"].cpu().view(torch.int16) == d["scale"].view(torch.int16))
    same_z = (pk["zero"].cpu().view(torch.int16) == d["zero"].view(torch.int16))
    assert (same_s & same_z).float().mean() > 0.999
    rows_same = (same_s & same_z).reshape(-1)
    q_gpu = pk["q"].cpu().reshape(-1, 32)
    q_ref = d["q"].reshape(-1, 32)
    assert torch.equal(q_gpu[rows_same], q_ref[rows_same])


def _ties_only(pk, ref):
    """Groups where (scale, zero) differ must be near-ties of the clip search; elsewhere the codes are identical.
    Returns the fraction of differing groups."""
    same = (pk["scale"].view(torch.int16) == ref["scale"].view(torch.int16)) & \
           (pk["zero"].view(torch.int16) == ref["zero"].view(torch.int16))
    flat = same.reshape(-1)
    qa, qb = pk["q"].reshape(-1, 32), ref["q"].reshape(-1, 32)
    assert torch.equal(qa[flat], qb[flat])
    return 1.0 - flat.float().mean().item()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantize_kernel_vs_torch_steps(dev, dtype):
    """The CUDA quantizer (group 64) against the same clip search as torch operations on the GPU
    (smelb.quant._quantize_slab): identical bytes except on near-ties of the candidates' squared errors. The input
    holds constant groups (zero range), one-outlier groups and a range of magnitudes."""
    from smelb import quant
    g = torch.Generator(device=dev).manual_seed(11)
    w = torch.randn(20, 96, 512, generator=g, device=dev) * 0.02
    w[0, :8] = 0.25                                   # constant groups: step clamps to 1e-8
    w[1, :8, ::64] = 3.0                               # one outlier per group
    w[2] *= 1e-4
    w[3] *= 50.0
    w = w.to(dtype)
    pk = quant.quantize_int4(w, 64)
    ref = quant._quantize_slab(w, 64, quant.CLIP_SEARCH)
    assert pk["q"].shape == ref["q"].shape and pk["scale"].dtype == torch.bfloat16
    assert _ties_only(pk, ref) < 1e-3
    # one candidate (no clip search), and the default tuple as a list
    pk1 = quant.quantize_int4(w, 64, clip_search=(1.0,))
    ref1 = quant._quantize_slab(w, 64, (1.0,))
    assert _ties_only(pk1, ref1) == 0.0
    assert _ties_only(quant.quantize_int4(w, 64, clip_search=list(quant.CLIP_SEARCH)), pk) == 0.0
    _status_ok()


def test_router_topk_bit_exact_given_logits(dev):
    """Given identical bf16 logits the routing indices are bit-exact (ties -> smaller expert id) and topv equals the
    oracle's renormalised weights cast to bf16 up to one bf16 ulp."""
    from smelb import _lib
    g = torch.Generator().manual_seed(7)
    T, E, K = 333, 256, 8
    logits = (torch.randn(T, E, generator=g) * 2).bfloat16()
    logits[:50, 10:20] = 1.5  # exact ties inside and at the top-k boundary
    logits[50:60] = 0.0       # all experts tied
    lg = logits.to(dev)
    probs = torch.empty(T, E, device=dev)
    topv = torch.empty(T, K, device=dev, dtype=torch.bfloat16)
    topi = torch.empty(T, K, device=dev, dtype=torch.int64)
    _lib.call("smelb_router_topk", lg.data_ptr(), E, T, E, K, probs.data_ptr(), topv.data_ptr(), 0, topi.data_ptr(),
              None, _lib.stream_ptr())
    p_ref, v_ref, i_ref = O.route_from_logits(logits.float(), K)
    assert torch.equal(topi.cpu(), i_ref)
    assert torch.allclose(probs.cpu(), p_ref, rtol=2e-6, atol=1e-9)
    diff = (topv.cpu().float() - v_ref.float()).abs()
    assert (diff <= v_ref.float().abs() * 2 ** -7).all()


@pytest.mark.parametrize("entry", ["smelb_dispatch_plan", "smelb_dispatch_plan_ws"])
def test_dispatch_plan_bit_exact(dev, golden, entry):
    """One-CTA plan and the many-CTA plan (the layer's) against the oracle's stable sort, bit for bit."""
    from smelb import _lib
    for T, K, E, seed in ((97, 4, 8, 0), (4092, 8, 256, 1), (1, 8, 256, 2), (3000, 2, 16, 3), (4092, 8, 256, 4),
                          (16384, 8, 128, 5)):
        g = torch.Generator().manual_seed(seed)
        topi = torch.randint(0, E, (T, K), generator=g)
        if seed == 3:
            topi[:, 0] = 5  # one very hot expert
        if seed == 4:  # Zipf-like skew: a few experts take most choices
            w = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** 1.1
            topi = torch.multinomial(w.expand(T, E), K, replacement=False, generator=g)
        sel = np.zeros(E, dtype=np.uint8)
        sel[[1, 5, E - 1]] = 1
        counts, gcounts, offsets, row_of, src_of = O.dispatch_padded(topi.numpy(), E, sel, 64)
        order, _, _ = O.dispatch(topi.numpy(), E)
        R = T * K + 3 * 64
        tg = topi.to(dev)
        b = {k: torch.full((n,), -7, dtype=torch.int32, device=dev) for k, n in
             (("counts", E), ("gcounts", E), ("offsets", E), ("row_of", T * K), ("src_of", R), ("total", 1))}
        order_d = torch.empty(T * K, dtype=torch.int64, device=dev)
        sel_d = torch.from_numpy(sel).to(dev)
        args = [tg.data_ptr(), T, K, E, sel_d.data_ptr(), 64, b["counts"].data_ptr(), b["gcounts"].data_ptr(),
                b["offsets"].data_ptr(), b["row_of"].data_ptr(), b["src_of"].data_ptr(), order_d.data_ptr(),
                b["total"].data_ptr()]
        if entry == "smelb_dispatch_plan_ws":
            ws = torch.full((148 * E,), -3, dtype=torch.int32, device=dev)
            args += [ws.data_ptr(), ws.numel()]
        _lib.call(entry, *args, _lib.stream_ptr())
        assert b["counts"].cpu().numpy().tolist() == counts.tolist()
        assert b["gcounts"].cpu().numpy().tolist() == gcounts.tolist()
        assert b["offsets"].cpu().numpy().tolist() == offsets.tolist()
        assert b["row_of"].cpu().numpy().tolist() == row_of.tolist()
        tot = int(b["total"].item())
        assert tot == src_of.size
        assert b["src_of"][:tot].cpu().numpy().tolist() == src_of.tolist()
        assert np.array_equal(order_d.cpu().numpy(), order)
    _status_ok()


def test_dispatch_matches_reference_golden(dev, golden):
    from smelb import _lib
    d = golden("dispatch.pt")
    T, K = d["topi"].shape
    E = d["E"]
    tg = d["topi"].to(dev)
    i32 = lambda n: torch.empty(n, dtype=torch.int32, device=dev)  # noqa: E731
    counts, gcounts, offsets, row_of, src_of, total = i32(E), i32(E), i32(E), i32(T * K), i32(T * K), i32(1)
    order = torch.empty(T * K, dtype=torch.int64, device=dev)
    _lib.call("smelb_dispatch_plan", tg.data_ptr(), T, K, E, None, 64, counts.data_ptr(), gcounts.data_ptr(),
              offsets.data_ptr(), row_of.data_ptr(), src_of.data_ptr(), order.data_ptr(), total.data_ptr(),
              _lib.stream_ptr())
    assert torch.equal(order.cpu(), d["order"])
    assert torch.equal(counts.cpu().long(), d["counts"])
    assert torch.equal((src_of.cpu().long() // K), d["tok"])
