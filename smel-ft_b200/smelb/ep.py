"""Expert parallelism for the MoE layer (smel/moe.py:255-263 partitioned by expert over the ranks of one box).

Rank p of P owns experts [p E/P, (p+1) E/P): its slice of the frozen int4 bank, its selected (LoRA) experts and
their LoRA factors. The router and the shared expert (with its LoRA) are replicated; every rank routes and combines
its own tokens. One call:

  1. route the rank's tokens over all E experts (the replicated router);
  2. plan the stable dispatch by expert id; experts are contiguous per rank, so the dispatch order is also grouped
     by destination rank (moe.py:216-223 order, unchanged);
  3. exchange per-expert row counts (all-to-all, E/P ints per peer), then the token rows themselves
     (all-to-all-v of bf16 H-vectors, NCCL over NVLink);
  4. every owner runs its experts on the rows it received, as K=1 tokens with routing weight 1 (the combine of that
     call is then the identity), through the same fused kernels as the single-GPU layer;
  5. the expert outputs travel back by the reverse all-to-all and are combined at the source in fp32, k order
     (moe.py:248-252), then the shared expert is added (moe.py:263).

Autograd mirrors it: the backward of each all-to-all is the reverse all-to-all, the owners produce dX rows for the
rows they received and the LoRA gradients of their selected experts (which stay on the owner). The shared expert's
LoRA gradients are per-rank partial sums; `allreduce_shared_grads` sums them (once per optimizer step).

The compute steps go through an `ops` object; the default runs the smelb kernels on CUDA tensors (no CPU path).
"""
import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .lora import ExpertsLoRA, LayerLoRA
from .moe import BF16Experts, Int4Experts, LayerExperts, _bf16, route, routed_experts, shared_mlp


# ------------------------------------------------------------------------------------------ sharding
def expert_range(E: int, rank: int, world: int):
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    n = E // world
    return rank * n, (rank + 1) * n


def shard_layer(ex: LayerExperts, lora_layer, rank: int, world: int):
    """(local LayerExperts, local LayerLoRA) of `rank`: the frozen-bank slice of its experts, its selected experts
    (local ids) and fresh Parameters holding its selected experts' LoRA factors; the shared LoRA is kept as is
    (replicated)."""
    e0, e1 = expert_range(ex.E, rank, world)
    fz = ex.frozen
    if isinstance(fz, Int4Experts):
        bank = Int4Experts({k: v[e0:e1] for k, v in fz.gu.items()}, {k: v[e0:e1] for k, v in fz.dn.items()},
                           fz.dtype)
    elif isinstance(fz, BF16Experts):
        bank = BF16Experts(fz.gate_up[e0:e1], fz.down[e0:e1])
    else:
        raise TypeError(f"shard_layer: unsupported bank {type(fz).__name__}")
    slots, loc_ids = [], []
    if ex.sel_ids is not None:
        for j, e in enumerate(ex.sel_ids.tolist()):
            if e0 <= e < e1:
                slots.append(j)
                loc_ids.append(e - e0)
    if slots:
        ex_loc = LayerExperts(bank, loc_ids, ex.sel_gate_up[slots], ex.sel_down[slots], ex.group, ex.act)
    else:
        ex_loc = LayerExperts(bank, None, None, None, ex.group, ex.act)
    lora_loc = None
    if lora_layer is not None:
        le = lora_layer.experts
        le_loc = None
        if le is not None and slots:
            H, I = le.A_gate.shape[2], le.B_gate.shape[1]
            le_loc = ExpertsLoRA(loc_ids, H, I, le.r, le.alpha).to(le.A_gate.device)
            with torch.no_grad():
                for n in ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down"):
                    getattr(le_loc, n).copy_(getattr(le, n)[slots])
        lora_loc = LayerLoRA(le_loc, lora_layer.shared)
    return ex_loc, lora_loc


def allreduce_shared_grads(lora_layer, group=None):
    """Sum the replicated shared-expert LoRA gradients over the ranks (once per optimizer step)."""
    if lora_layer is None or lora_layer.shared is None:
        return
    for p in lora_layer.shared.parameters():
        if p.grad is not None:
            dist.all_reduce(p.grad, group=group)


# ------------------------------------------------------------------------------------------ exchange
class _AllToAll(torch.autograd.Function):
    """Rows exchange: `in_splits[p]` rows of x go to rank p, `out_splits[p]` rows arrive from rank p (in rank
    order). The backward is the reverse exchange."""

    @staticmethod
    def forward(ctx, x, out_splits, in_splits, group):
        ctx.splits = (out_splits, in_splits)
        ctx.group = group
        out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out_splits, in_splits = ctx.splits
        gi = g.new_empty((sum(in_splits),) + tuple(g.shape[1:]))
        dist.all_to_all_single(gi, g.contiguous(), in_splits, out_splits, group=ctx.group)
        return gi, None, None, None


# ------------------------------------------------------------------------------------------ CUDA ops
class _Plan:
    def __init__(self, counts, row_of, src_of, order, total, R):
        self.counts, self.row_of, self.src_of, self.order, self.total, self.R = counts, row_of, src_of, order, total, R


class _GatherFn(torch.autograd.Function):
    """xs[row] = x[src_of[row] // K] (moe.py:221); backward dx[t] = sum_k dxs[row_of[t, k]] (fp32, k order)."""

    @staticmethod
    def forward(ctx, x, plan, K):
        T, H = x.shape
        xs = torch.empty(plan.R, H, dtype=torch.bfloat16, device=x.device)
        _lib.call("smelb_gather_rows", _lib.ptr(x), H, K, _lib.ptr(plan.src_of), _lib.ptr(plan.total), plan.R,
                  _lib.ptr(xs), _lib.stream_ptr(x.device))
        ctx.plan, ctx.K, ctx.T = plan, K, T
        return xs

    @staticmethod
    def backward(ctx, g):
        g = g.to(torch.bfloat16).contiguous()
        H = g.shape[1]
        dx = torch.empty(ctx.T, H, dtype=torch.bfloat16, device=g.device)
        _lib.call("smelb_gather_rows_bwd", _lib.ptr(g), _lib.ptr(ctx.plan.row_of), ctx.T, ctx.K, H, _lib.ptr(dx),
                  _lib.stream_ptr(g.device))
        return dx, None, None


class _CombineFn(torch.autograd.Function):
    """out[t] = bf16(sum_k fp32(y[row_of[t, k]]) * fp32(topv[t, k])) (moe.py:248-252) and its backward."""

    @staticmethod
    def forward(ctx, y, topv, plan, K):
        y = y.contiguous()
        T = topv.shape[0]
        H = y.shape[1]
        f32 = topv.dtype == torch.float32
        out = torch.empty(T, H, dtype=torch.bfloat16, device=y.device)
        _lib.call("smelb_combine_fwd", _lib.ptr(y), _lib.ptr(plan.row_of), _lib.ptr(topv), 1 if f32 else 0, T, K, H,
                  _lib.ptr(out), _lib.stream_ptr(y.device))
        ctx.save_for_backward(y, topv)
        ctx.plan, ctx.K = plan, K
        return out

    @staticmethod
    def backward(ctx, g):
        y, topv = ctx.saved_tensors
        g = g.to(torch.bfloat16).contiguous()
        f32 = topv.dtype == torch.float32
        dy = torch.empty_like(y)
        dtopv = torch.empty_like(topv)
        _lib.call("smelb_combine_bwd", _lib.ptr(g), _lib.ptr(y), _lib.ptr(ctx.plan.src_of), _lib.ptr(ctx.plan.total),
                  ctx.plan.R, _lib.ptr(topv), 1 if f32 else 0, ctx.K, y.shape[1], _lib.ptr(dy), _lib.ptr(dtopv),
                  _lib.stream_ptr(g.device))
        return dy, dtopv, None, None


class CudaOps:
    """The compute steps of an expert-parallel layer call on the smelb kernels."""

    def route(self, x, gate_w, top_k):
        return route(x, gate_w, top_k)

    def plan(self, topi, E):
        T, K = topi.shape
        dev = topi.device
        R = T * K
        i32 = lambda n: torch.empty(n, dtype=torch.int32, device=dev)  # noqa: E731
        counts, gcounts, offsets, row_of, src_of, total = i32(E), i32(E), i32(E), i32(R), i32(R), i32(1)
        order = torch.empty(R, dtype=torch.int64, device=dev)
        ws = i32(148 * E)
        topi = topi.contiguous()
        _lib.call("smelb_dispatch_plan_ws", _lib.ptr(topi), T, K, E, None, 1, _lib.ptr(counts), _lib.ptr(gcounts),
                  _lib.ptr(offsets), _lib.ptr(row_of), _lib.ptr(src_of), _lib.ptr(order), _lib.ptr(total),
                  _lib.ptr(ws), ws.numel(), _lib.stream_ptr(dev))
        return _Plan(counts, row_of, src_of, order, total, R)

    def gather(self, x, plan, K):
        return _GatherFn.apply(_bf16(x, "moe_forward_ep: x"), plan, K)

    def combine(self, y, topv, plan, K):
        return _CombineFn.apply(y, topv, plan, K)

    def experts(self, x_recv, topi_loc, ex_loc, lora_loc):
        lora_ex = lora_loc.experts if lora_loc is not None else None
        topv = torch.ones(x_recv.shape[0], 1, dtype=torch.bfloat16, device=x_recv.device)
        return routed_experts(x_recv, topv, topi_loc, ex_loc, lora_ex)

    def shared(self, x, W, lora_loc):
        return shared_mlp(x, W, lora_loc.shared if lora_loc is not None else None)

    def counts_of(self, plan):
        return plan.counts


# ------------------------------------------------------------------------------------------ the layer
def moe_forward_ep(x2d, W, ex_loc, top_k, lora_loc=None, group=None, ops=None, stats=None, n_experts=None):
    """moe_forward (moe.py:255-263) with the routed experts partitioned over the ranks of `group`.

    x2d: this rank's tokens [T, H]; W: the replicated router / shared-expert tensors; ex_loc, lora_loc: this rank's
    experts and LoRA (from shard_layer). Returns this rank's [T, H] output, differentiable w.r.t. x2d, the local
    LoRA parameters and the shared LoRA parameters."""
    ops = ops or CudaOps()
    P = dist.get_world_size(group)
    E = n_experts if n_experts is not None else W["mlp.gate.weight"].shape[0]
    E_loc = E // P
    if E_loc * P != E:
        raise ValueError(f"{E} experts do not split evenly over {P} ranks")
    probs, topv, topi = ops.route(x2d, W["mlp.gate.weight"], top_k)
    if stats is not None:
        stats(probs, topv, topi)
    plan = ops.plan(topi, E)
    counts = ops.counts_of(plan)
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts.contiguous(), group=group)
    ch = torch.stack((counts, recv_counts)).cpu().numpy().astype(np.int64)  # one small copy: the row splits
    send_splits = ch[0].reshape(P, E_loc).sum(1).tolist()
    recv_splits = ch[1].reshape(P, E_loc).sum(1).tolist()
    xs = ops.gather(x2d, plan, top_k)
    x_recv = _AllToAll.apply(xs, recv_splits, send_splits, group)
    # local expert id of every received row: by source rank, then by expert (the sender's dispatch order)
    ids = np.repeat(np.tile(np.arange(E_loc), P), ch[1])
    topi_loc = torch.from_numpy(ids).to(x_recv.device).view(-1, 1)
    if x_recv.shape[0]:
        y_recv = ops.experts(x_recv, topi_loc, ex_loc, lora_loc)
    else:
        y_recv = x_recv * 0
    y_back = _AllToAll.apply(y_recv, send_splits, recv_splits, group)
    out = ops.combine(y_back, topv, plan, top_k)
    return out + ops.shared(x2d, W, lora_loc)
