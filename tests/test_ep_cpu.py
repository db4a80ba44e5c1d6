"""Expert parallelism on the CPU: the placement and sharding logic of smelb/ep.py, and the exchange protocol that
csrc/ep.cu implements, modelled step by step in torch on two gloo ranks and checked against one single-process oracle
layer (oracle/moe_oracle.py) over both ranks' tokens.

The model keeps the kernels' data flow and orders: per destination the tokens with an expert there, once each, in
token order, with the row's entries (local expert, k, weight) in k order; the owner numbers the entries in (source,
row, slot) order, runs its experts on them and returns per row the weighted sum of its entries; the source adds the
owners' rows in rank order plus the shared expert. Backward: the gradient rows go to the owners, which form
dY = g * w and d w = g . y per entry, run the expert backward and return per row the summed dX of its entries and the
d w of each entry, which the source maps back to its (t, k) by the row's slot order. The model computes in fp64 and
the oracle's weighted combine in fp32 (as the reference's), so they agree to fp32 rounding (1e-6), while a misrouted
row or entry would be an O(1) error; the kernels' bf16 rounding is checked against the single-GPU layer on the GPU
(tests/test_gpu_ep.py)."""
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "smel-ft_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

H, E, K, I, S, T, R_LORA, ALPHA = 64, 8, 3, 64, 64, 40, 8, 16.0
SEL = [1, 6, 3]
NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")
DT = torch.float64


# ------------------------------------------------------------------------------------------ placement
def test_balanced_placement_is_even_and_balanced():
    from smelb import ep
    loads = [100, 1, 1, 1, 90, 2, 3, 80, 5, 5, 7, 1]
    pl = ep.balanced_placement(loads, 3)
    assert sorted(e for p in pl for e in p) == list(range(12)) and all(len(p) == 4 for p in pl)
    per = [sum(loads[e] for e in p) for p in pl]
    contiguous = [sum(loads[e] for e in p) for p in ep.contiguous_placement(12, 3)]
    assert max(per) - min(per) < max(contiguous) - min(contiguous)
    assert max(per) <= max(loads) + 10  # the three hot experts land on three different ranks
    assert ep.balanced_placement(loads, 3) == pl  # deterministic
    with pytest.raises(ValueError):
        ep.balanced_placement(loads, 5)



def test_balanced_placement_weighs_expert_cost():
    """Config-2-like loads over 8 ranks: 12 hot selected experts (half the rows) and 244 frozen ones, each frozen
    expert adding a fixed cost per token tile (expert_costs). Balancing that cost keeps every rank within 2% of the
    mean (rows alone leave more than 3%), every rank keeping E / world experts."""
    from smelb import ep
    import random

    class _Ex:  # the one field expert_costs reads
        pass
    rnd = random.Random(3)
    E, world = 256, 8
    sel = list(range(0, 24, 2))
    loads = [rnd.randint(20, 220) for _ in range(E)]
    for e in sel:
        loads[e] = 1400 + rnd.randint(0, 200)
    ex = _Ex()
    ex.sel_ids = torch.tensor(sel)
    costs = ep.expert_costs(ex, loads)
    assert all(costs[e] == loads[e] for e in sel)
    assert all(costs[e] > loads[e] for e in range(E) if e not in sel)

    def spread(pl):
        c = [sum(costs[e] for e in ids) for ids in pl]
        return max(c) / (sum(c) / len(c))
    rows_only = ep.balanced_placement(loads, world)
    weighted = ep.balanced_placement(loads, world, costs)
    assert all(len(ids) == E // world for ids in weighted)
    assert sorted(e for ids in weighted for e in ids) == list(range(E))
    assert spread(weighted) < 1.02 < spread(rows_only)

def test_shard_layer_takes_the_placed_experts():
    import smelb
    from smelb import ep
    E_, H_, I_ = 6, 64, 64
    q = torch.arange(E_).view(E_, 1, 1).expand(E_, 2 * I_, H_ // 2).to(torch.uint8).contiguous()
    s = torch.ones(E_, 2 * I_, 1, dtype=torch.bfloat16)
    qd = torch.arange(E_).view(E_, 1, 1).expand(E_, H_, I_ // 2).to(torch.uint8).contiguous()
    sd = torch.ones(E_, H_, 1, dtype=torch.bfloat16)
    bank = smelb.Int4Experts({"q": q, "scale": s, "zero": s}, {"q": qd, "scale": sd, "zero": sd})
    sel = [4, 1]
    ex = smelb.LayerExperts(bank, sel, torch.zeros(2, 2 * I_, H_), torch.zeros(2, H_, I_))
    lex = smelb.ExpertsLoRA(sel, H_, I_, 8, 16.0)
    lsh = smelb.MLPLoRA(H_, 32, 8, 16.0)
    with torch.no_grad():
        lex.A_gate[0].fill_(4.0)
        lex.A_gate[1].fill_(1.0)
    pl = [[0, 4, 5], [1, 2, 3]]
    sh = ep.shard_layer(ex, smelb.LayerLoRA(lex, lsh), 0, 2, pl)
    assert [int(v) for v in sh.ex.frozen.gu["q"][:, 0, 0]] == [0, 4, 5]
    assert sh.ex.sel_ids.tolist() == [1] and float(sh.lora.experts.A_gate.detach()[0, 0, 0]) == 4.0
    assert sh.lora.shared is lsh
    sh1 = ep.shard_layer(ex, smelb.LayerLoRA(lex, lsh), 1, 2, pl)
    assert sh1.ex.sel_ids.tolist() == [0] and float(sh1.lora.experts.A_gate.detach()[0, 0, 0]) == 1.0
    with pytest.raises(ValueError):
        ep.shard_layer(ex, None, 0, 2, [[0, 1], [2, 3]])


# ------------------------------------------------------------------------------------------ protocol model
def _data():
    from oracle import moe_oracle as O
    g = torch.Generator().manual_seed(0)
    rnd = lambda *s, std=0.02: torch.randn(*s, generator=g, dtype=DT) * std  # noqa: E731
    x = rnd(2 * T, H, std=1.0)
    W = {"mlp.gate.weight": rnd(E, H) * 10, "mlp.shared_expert.gate_proj.weight": rnd(S, H),
         "mlp.shared_expert.up_proj.weight": rnd(S, H), "mlp.shared_expert.down_proj.weight": rnd(H, S),
         "mlp.shared_expert_gate.weight": rnd(1, H)}
    gu, dn = rnd(E, 2 * I, H), rnd(E, H, I)
    qg, qd = O.quantize_int4(gu.float()), O.quantize_int4(dn.float())
    bank_gu = O.dequant_int4(qg["q"], qg["scale"], qg["zero"]).to(DT)
    bank_dn = O.dequant_int4(qd["q"], qd["scale"], qd["zero"]).to(DT)
    shapes = {"A_gate": (R_LORA, H), "B_gate": (I, R_LORA), "A_up": (R_LORA, H), "B_up": (I, R_LORA),
              "A_down": (R_LORA, I), "B_down": (H, R_LORA)}
    lora_ex = {n: rnd(len(SEL), *shapes[n], std=0.1) for n in NAMES}
    lora_sh = {n: rnd(*([S if d == I else d for d in shapes[n]]), std=0.1) for n in NAMES}
    gy = rnd(2 * T, H, std=1.0)
    return x, W, bank_gu, bank_dn, gu[SEL], dn[SEL], lora_ex, lora_sh, gy


def _exchange(payload):
    """payload[d] for every destination d -> the payloads every source sent to this rank, in source order."""
    got = [None] * dist.get_world_size()
    dist.all_gather_object(got, payload)
    return [got[s][dist.get_rank()] for s in range(len(got))]


def _worker(rank, world, port, errq):
    try:
        for p in (ROOT, os.path.join(ROOT, "smel-ft_b200")):
            sys.path.insert(0, p)
        from oracle import moe_oracle as O
        from smelb import ep
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        x, W, bank_gu, bank_dn, sel_gu, sel_dn, lora_ex, lora_sh, gy = _data()
        scale = ALPHA / R_LORA
        # single-process reference over both ranks' tokens
        xr = x.clone().requires_grad_(True)
        lex = {n: v.clone().requires_grad_(True) for n, v in lora_ex.items()}
        lsh = {n: v.clone().requires_grad_(True) for n, v in lora_sh.items()}
        ref, _, _, topi_all = O.moe_layer(xr, W, bank_gu, bank_dn, K, SEL, sel_gu, sel_dn, dict(lex, scale=scale),
                                          dict(lsh, scale=scale))
        (ref * gy).sum().backward()
        loads = torch.bincount(topi_all.reshape(-1), minlength=E).tolist()
        pl = ep.balanced_placement(loads, world)
        owner = {e: r for r, ids in enumerate(pl) for e in ids}
        local = {e: j for ids in pl for j, e in enumerate(ids)}
        mine_e = pl[rank]
        sel_here = [j for j, e in enumerate(SEL) if owner[e] == rank]
        lloc = {n: lora_ex[n][sel_here].clone().requires_grad_(True) for n in NAMES}
        slot_of = {local[SEL[j]]: i for i, j in enumerate(sel_here)}
        sl = slice(rank * T, (rank + 1) * T)
        xl = x[sl].clone().requires_grad_(True)
        # ---- source: route, plan (one row per token and destination, token order; entries in k order)
        probs = torch.softmax(F.linear(xl, W["mlp.gate.weight"]), -1)
        topi = O.topk_stable(probs, K)
        top = probs.gather(1, topi)
        topv = top / top.sum(-1, keepdim=True)
        assert any(owner[int(e)] != rank for e in topi.reshape(-1)), "no cross-rank traffic in the test data"
        rows = [[] for _ in range(world)]      # per destination: (token, [(local id, k, w)])
        pos, slot_j = {}, {}
        for t in range(T):
            for d in range(world):
                ent = [(local[int(topi[t, k])], k, float(topv[t, k])) for k in range(K) if owner[int(topi[t, k])] == d]
                if ent:
                    pos[(t, d)] = len(rows[d])
                    for j, (_, k, _) in enumerate(ent):
                        slot_j[(t, k)] = j
                    rows[d].append((t, ent))
        recv = _exchange([[(xl[t].detach(), ent) for t, ent in rows[d]] for d in range(world)])
        # ---- owner: entries in (source, row, slot) order, experts, one weighted partial row per received row
        xrecv = [torch.stack([r[0] for r in src]).requires_grad_(True) if src else None for src in recv]
        entries = [(s, i, le, w) for s, src in enumerate(recv) for i, (_, ent) in enumerate(src) for le, _, w in ent]
        y_ent = []
        for s, i, le, w in entries:
            xe = xrecv[s][i:i + 1]
            if le in slot_of:
                j = slot_of[le]
                Lj = dict({n: lloc[n][j] for n in NAMES}, scale=scale)
                ye = O.mlp(xe, sel_gu[sel_here[j]][:I], sel_gu[sel_here[j]][I:], sel_dn[sel_here[j]], Lj, "silu")
            else:
                e = mine_e[le]
                gg, uu = (xe @ bank_gu[e].t()).chunk(2, dim=-1)
                ye = (O.act(gg, "silu") * uu) @ bank_dn[e].t()
            y_ent.append(ye[0])
        part = [[torch.zeros(H, dtype=DT) for _ in src] for src in recv]
        for (s, i, le, w), ye in zip(entries, y_ent):
            part[s][i] = part[s][i] + w * ye.detach()
        back = _exchange(part)
        # ---- source: owners' rows in rank order plus the shared expert
        pre = "mlp.shared_expert."
        lsh_loc = {n: v.clone().requires_grad_(True) for n, v in lora_sh.items()}  # replicated shared LoRA
        sh = O.mlp(xl, W[pre + "gate_proj.weight"], W[pre + "up_proj.weight"], W[pre + "down_proj.weight"],
                   dict(lsh_loc, scale=scale), "silu") * torch.sigmoid(F.linear(xl, W["mlp.shared_expert_gate.weight"]))
        routed = torch.stack([sum((back[d][pos[(t, d)]] for d in range(world) if (t, d) in pos),
                                  torch.zeros(H, dtype=DT)) for t in range(T)])
        out = routed + sh.detach()
        g = gy[sl]
        # ---- backward: gradient rows to the owners (same rows), dY = g w and d w = g . y per entry
        grecv = _exchange([[g[t] for t, _ in rows[d]] for d in range(world)])
        dw = []
        ys = [ye for ye in y_ent]
        dys = []
        for (s, i, le, w), ye in zip(entries, y_ent):
            gr = grecv[s][i]
            dys.append(gr * w)
            dw.append(float((gr * ye.detach()).sum()))
        if ys:
            torch.autograd.backward(ys, dys)
        dx_part = [xr_.grad if xr_ is not None else None for xr_ in xrecv]
        dw_rows = [[[] for _ in src] for src in recv]
        for (s, i, le, w), v in zip(entries, dw):
            dw_rows[s][i].append(v)
        back_b = _exchange([[(dx_part[s][i], dw_rows[s][i]) for i in range(len(recv[s]))] if recv[s] else []
                            for s in range(world)])
        dx_routed = torch.stack([sum((back_b[d][pos[(t, d)]][0] for d in range(world) if (t, d) in pos),
                                     torch.zeros(H, dtype=DT)) for t in range(T)])
        dtopv = torch.zeros(T, K, dtype=DT)
        for t in range(T):
            for k in range(K):
                d = owner[int(topi[t, k])]
                dtopv[t, k] = back_b[d][pos[(t, d)]][1][slot_j[(t, k)]]
        # the router and the shared expert by autograd, with the returned d topv and g
        ((topv * dtopv).sum() + (sh * g).sum()).backward()
        dx = dx_routed + xl.grad
        for n in NAMES:
            dist.all_reduce(lsh_loc[n].grad)
        checks = [("out", out, ref[sl]), ("dx", dx, xr.grad[sl])]
        checks += [(f"sel {n}", lloc[n].grad, lex[n].grad[sel_here]) for n in NAMES if sel_here]
        checks += [(f"shared {n}", lsh_loc[n].grad, lsh[n].grad) for n in NAMES]
        for name, a, b in checks:
            e = O.rel_err(a, b)
            assert e < 1e-6, f"rank {rank} {name}: rel err {e:.3e}"
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(f"rank {rank}: {traceback.format_exc()}")
        raise


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_protocol_two_gloo_ranks_match_single_layer():
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
