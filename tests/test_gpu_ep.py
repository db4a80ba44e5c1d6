"""Expert parallelism on two GPUs (NCCL): smelb.ep.moe_forward_ep over two ranks, each holding half of the experts,
against the single-GPU fused layer (smelb.moe_forward) on the union of the tokens: output, dX and the LoRA
gradients (owner-side for the selected experts, all-reduced for the shared expert) within the tolerance of the
other layer tests (max relative error 2e-2, cosine 0.9999). Skipped with fewer than two GPUs."""
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu
REL, COS = 2e-2, 0.9999
NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")


def _worker(rank, world, port, errq, T):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "smel-ft_b200"))
        from oracle import moe_oracle as O
        import smelb
        from smelb import ep
        from smelb.synth import qwen_layer
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        L = qwen_layer(T=world * T, H=512, E=32, K=4, I=256, S=256, n_sel=4, r=16, seed=3, device=dev)
        W, ex, lora, x = L["W"], L["ex"], L["lora"], L["x"]
        gy = torch.randn(x.shape, generator=torch.Generator(device=dev).manual_seed(5), device=dev).bfloat16()
        # single-GPU reference over all tokens
        xr = x.detach().clone().requires_grad_(True)
        ref = smelb.moe_forward(xr, W, ex, 4, lora)
        ref.backward(gy)
        ref_sel = {n: getattr(lora.experts, n).grad.clone() for n in NAMES}
        ref_sh = {n: getattr(lora.shared, n).grad.clone() for n in NAMES}
        for p in lora.parameters():
            p.grad = None
        # expert parallel: this rank's tokens and half of the experts
        ex_loc, lora_loc = ep.shard_layer(ex, lora, rank, world)
        e0, e1 = ep.expert_range(ex.E, rank, world)
        slots = [j for j, e in enumerate(ex.sel_ids.tolist()) if e0 <= e < e1]
        sl = slice(rank * T, (rank + 1) * T)
        xl = x[sl].detach().clone().requires_grad_(True)
        out = ep.moe_forward_ep(xl, W, ex_loc, 4, lora_loc)
        out.backward(gy[sl])
        ep.allreduce_shared_grads(lora_loc)
        checks = [("out", out, ref[sl]), ("dx", xl.grad, xr.grad[sl])]
        if slots:
            checks += [(f"sel {n}", getattr(lora_loc.experts, n).grad, ref_sel[n][slots]) for n in NAMES]
        checks += [(f"shared {n}", getattr(lora_loc.shared, n).grad, ref_sh[n]) for n in NAMES]
        bad = []
        for name, a, b in checks:
            e, c = O.rel_err(a.float().cpu(), b.float().cpu()), O.cosine(a.float().cpu(), b.float().cpu())
            if not (e <= REL and c >= COS):
                bad.append(f"{name}: rel err {e:.3e} cosine {c:.6f}")
        assert not bad, f"rank {rank}: " + "; ".join(bad)
        assert smelb.read_status() == 0
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(f"rank {rank}: {traceback.format_exc()}")
        raise


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_two_gpus_match_single_gpu_layer():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errq, 512)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not errs, "\n".join(errs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
