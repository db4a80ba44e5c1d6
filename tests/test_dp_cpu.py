"""Data parallelism (smelb/dp.py): two gloo ranks on the CPU, each running the layer on its own half of the tokens
(the compute is the oracle layer of oracle/moe_oracle.py; the CUDA kernels do not run on the CPU). After
GradAllReduce the LoRA gradients on both ranks equal those of one single-process layer over all the tokens
(gradients of a sum over tokens are the sum of the per-half gradients)."""
import os
import socket
import sys
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
H, E, K, I, S, T, R_LORA, ALPHA = 64, 8, 2, 64, 64, 40, 8, 16.0
SEL = [1, 6]
NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")


def _data():
    from oracle import moe_oracle as O
    g = torch.Generator().manual_seed(1)
    rnd = lambda *s, std=0.02: torch.randn(*s, generator=g) * std  # noqa: E731
    x = rnd(2 * T, H, std=1.0)
    W = {"mlp.gate.weight": rnd(E, H) * 10, "mlp.shared_expert.gate_proj.weight": rnd(S, H),
         "mlp.shared_expert.up_proj.weight": rnd(S, H), "mlp.shared_expert.down_proj.weight": rnd(H, S),
         "mlp.shared_expert_gate.weight": rnd(1, H)}
    gu, dn = rnd(E, 2 * I, H), rnd(E, H, I)
    qg, qd = O.quantize_int4(gu), O.quantize_int4(dn)
    bank_gu = O.dequant_int4(qg["q"], qg["scale"], qg["zero"])
    bank_dn = O.dequant_int4(qd["q"], qd["scale"], qd["zero"])
    shapes = {"A_gate": (R_LORA, H), "B_gate": (I, R_LORA), "A_up": (R_LORA, H), "B_up": (I, R_LORA),
              "A_down": (R_LORA, I), "B_down": (H, R_LORA)}
    lora_ex = {n: rnd(len(SEL), *shapes[n], std=0.1) for n in NAMES}
    lora_sh = {n: rnd(*([S if d == I else d for d in shapes[n]]), std=0.1) for n in NAMES}
    gy = rnd(2 * T, H, std=1.0)
    return x, W, bank_gu, bank_dn, gu[SEL], dn[SEL], lora_ex, lora_sh, gy


def _grads(O, x, W, bank_gu, bank_dn, sel_gu, sel_dn, lora_ex, lora_sh, gy):
    lex = {n: v.clone().requires_grad_(True) for n, v in lora_ex.items()}
    lsh = {n: v.clone().requires_grad_(True) for n, v in lora_sh.items()}
    out, _, _, _ = O.moe_layer(x, W, bank_gu, bank_dn, K, SEL, sel_gu, sel_dn, dict(lex, scale=ALPHA / R_LORA),
                               dict(lsh, scale=ALPHA / R_LORA))
    (out * gy).sum().backward()
    return lex, lsh


def _worker(rank, world, port, errq):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "smel-ft_b200"))
        from oracle import moe_oracle as O
        from smelb import dp
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        x, W, bank_gu, bank_dn, sel_gu, sel_dn, lora_ex, lora_sh, gy = _data()
        ref_ex, ref_sh = _grads(O, x, W, bank_gu, bank_dn, sel_gu, sel_dn, lora_ex, lora_sh, gy)
        sl = slice(rank * T, (rank + 1) * T)
        mine_ex, mine_sh = _grads(O, x[sl], W, bank_gu, bank_dn, sel_gu, sel_dn, lora_ex, lora_sh, gy[sl])
        params = list(mine_ex.values()) + list(mine_sh.values())
        sync = dp.GradAllReduce(params)
        sync()
        sync()  # a second call reuses the buffer; summing already-summed gradients doubles them
        for n in NAMES:
            for name, a, b in ((f"sel {n}", mine_ex[n].grad, ref_ex[n].grad), (f"shared {n}", mine_sh[n].grad,
                                                                               ref_sh[n].grad)):
                e = O.rel_err(a, 2 * b)
                assert e < 1e-5, f"rank {rank} {name}: rel err {e:.3e}"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(f"rank {rank}: {traceback.format_exc()}")
        raise


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_data_parallel_two_gloo_ranks_sum_lora_grads():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not errs, "\n".join(errs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
