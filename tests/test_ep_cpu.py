"""Expert-parallel orchestration (smelb/ep.py: routing, per-expert count exchange, row all-to-all and its reverse,
combine, owner-side LoRA gradients, shared-LoRA all-reduce) on two gloo ranks on the CPU.

The compute steps are injected as oracle functions (the CUDA kernels do not run on the CPU); the test checks each
rank's output, dX and the LoRA gradients against one single-process oracle layer (oracle/moe_oracle.py) over both
ranks' tokens, i.e. that the partitioned exchange reproduces smel/moe.py:255-263 on the union of the tokens."""
import os
import socket
import sys
import traceback

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

H, E, K, I, S, T, R_LORA, ALPHA = 64, 8, 2, 64, 64, 48, 8, 16.0
SEL = [1, 6]  # one selected (LoRA) expert on each of the two ranks
NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")


def _data():
    from oracle import moe_oracle as O
    g = torch.Generator().manual_seed(0)
    rnd = lambda *s, std=0.02: torch.randn(*s, generator=g) * std  # noqa: E731
    x = rnd(2 * T, H, std=1.0)
    W = {"mlp.gate.weight": rnd(E, H) * 10, "mlp.shared_expert.gate_proj.weight": rnd(S, H),
         "mlp.shared_expert.up_proj.weight": rnd(S, H), "mlp.shared_expert.down_proj.weight": rnd(H, S),
         "mlp.shared_expert_gate.weight": rnd(1, H)}
    gu, dn = rnd(E, 2 * I, H), rnd(E, H, I)
    qg, qd = O.quantize_int4(gu), O.quantize_int4(dn)
    bank_gu = O.dequant_int4(qg["q"], qg["scale"], qg["zero"])
    bank_dn = O.dequant_int4(qd["q"], qd["scale"], qd["zero"])
    sel_gu, sel_dn = gu[SEL], dn[SEL]
    shapes = {"A_gate": (R_LORA, H), "B_gate": (I, R_LORA), "A_up": (R_LORA, H), "B_up": (I, R_LORA),
              "A_down": (R_LORA, I), "B_down": (H, R_LORA)}
    lora_ex = {n: rnd(len(SEL), *shapes[n], std=0.1) for n in NAMES}
    lora_sh = {n: rnd(*([S if d == I else d for d in shapes[n]]), std=0.1) for n in NAMES}
    gy = rnd(2 * T, H, std=1.0)
    return x, W, bank_gu, bank_dn, sel_gu, sel_dn, lora_ex, lora_sh, gy


class OracleOps:
    """The expert-parallel compute steps as oracle functions (test infrastructure)."""

    def __init__(self, W, lora_sh):
        from oracle import moe_oracle as O
        self.O, self.W, self.lora_sh = O, W, lora_sh

    def route(self, x, gate_w, top_k):
        probs = torch.softmax(F.linear(x, gate_w), dim=-1, dtype=torch.float32)
        topi = self.O.topk_stable(probs, top_k)
        top = probs.gather(1, topi)
        return probs, (top / top.sum(-1, keepdim=True)).to(x.dtype), topi

    def plan(self, topi, E_):
        order, tok, counts = self.O.dispatch(topi.numpy(), E_)
        row_of = np.empty_like(order)
        row_of[order] = np.arange(order.shape[0])
        return {"tok": tok, "row_of": row_of, "counts": torch.from_numpy(counts.astype(np.int64))}

    def counts_of(self, plan):
        return plan["counts"]

    def gather(self, x, plan, top_k):
        return x[torch.from_numpy(plan["tok"])]

    def combine(self, y, topv, plan, top_k):
        yk = y[torch.from_numpy(plan["row_of"])].view(topv.shape[0], top_k, y.shape[1])
        return (yk.float() * topv.float().unsqueeze(-1)).sum(1).to(y.dtype)

    def experts(self, x_recv, topi_loc, ex_loc, lora_loc):
        O = self.O
        ids = topi_loc.view(-1)
        out = x_recv.new_zeros(x_recv.shape)
        for e in range(ex_loc["E"]):
            rows = (ids == e).nonzero().view(-1)
            if rows.numel() == 0:
                continue
            xe = x_recv[rows]
            if e in ex_loc["slot"]:
                j = ex_loc["slot"][e]
                L = dict({n: lora_loc[n][j] for n in NAMES}, scale=ALPHA / R_LORA)
                ye = O.mlp(xe, ex_loc["sel_gu"][j][:I], ex_loc["sel_gu"][j][I:], ex_loc["sel_dn"][j], L, "silu")
            else:
                g, u = (xe @ ex_loc["gu"][e].t()).chunk(2, dim=-1)
                ye = (O.act(g, "silu") * u) @ ex_loc["dn"][e].t()
            out = out.index_put((rows,), ye)
        return out

    def shared(self, x, W, lora_loc):
        O, pre = self.O, "mlp.shared_expert."
        L = dict(self.lora_sh, scale=ALPHA / R_LORA)
        sh = O.mlp(x, W[pre + "gate_proj.weight"], W[pre + "up_proj.weight"], W[pre + "down_proj.weight"], L, "silu")
        return sh * torch.sigmoid(F.linear(x, W["mlp.shared_expert_gate.weight"]))


def _worker(rank, world, port, errq):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "smel-ft_b200"))
        from oracle import moe_oracle as O
        from smelb import ep
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        x, W, bank_gu, bank_dn, sel_gu, sel_dn, lora_ex, lora_sh, gy = _data()
        # single-process reference over both ranks' tokens
        xr = x.clone().requires_grad_(True)
        lex = {n: v.clone().requires_grad_(True) for n, v in lora_ex.items()}
        lsh = {n: v.clone().requires_grad_(True) for n, v in lora_sh.items()}
        ref, _, _, topi = O.moe_layer(xr, W, bank_gu, bank_dn, K, SEL, sel_gu, sel_dn,
                                      dict(lex, scale=ALPHA / R_LORA), dict(lsh, scale=ALPHA / R_LORA))
        mine = topi[rank * T:(rank + 1) * T]
        assert bool((mine < E // 2).any()) and bool((mine >= E // 2).any()), "no cross-rank traffic in the test data"
        (ref * gy).sum().backward()
        # this rank: tokens [rank T, (rank+1) T), experts [rank E/2, (rank+1) E/2)
        e0, e1 = ep.expert_range(E, rank, world)
        slots = [j for j, e in enumerate(SEL) if e0 <= e < e1]
        ex_loc = {"E": e1 - e0, "gu": bank_gu[e0:e1], "dn": bank_dn[e0:e1], "sel_gu": sel_gu[slots],
                  "sel_dn": sel_dn[slots], "slot": {SEL[j] - e0: i for i, j in enumerate(slots)}}
        lloc = {n: lora_ex[n][slots].clone().requires_grad_(True) for n in NAMES}
        lsh_r = {n: v.clone().requires_grad_(True) for n, v in lora_sh.items()}
        ops = OracleOps(W, lsh_r)
        xl = x[rank * T:(rank + 1) * T].clone().requires_grad_(True)
        out = ep.moe_forward_ep(xl, W, ex_loc, K, lloc, ops=ops, n_experts=E)
        (out * gy[rank * T:(rank + 1) * T]).sum().backward()
        for n in NAMES:  # the replicated shared LoRA: per-rank partial gradients, summed over the ranks
            dist.all_reduce(lsh_r[n].grad)
        sl = slice(rank * T, (rank + 1) * T)
        checks = [("out", out, ref[sl]), ("dx", xl.grad, xr.grad[sl])]
        checks += [(f"sel {n}", lloc[n].grad, lex[n].grad[slots]) for n in NAMES]
        checks += [(f"shared {n}", lsh_r[n].grad, lsh[n].grad) for n in NAMES]
        for name, a, b in checks:
            e = O.rel_err(a, b)
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


def test_expert_parallel_two_gloo_ranks_match_single_layer():
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
