"""Expert parallelism for the MoE layer: smel/moe.py:255-263 partitioned by expert over the P ranks (GPUs) of one box.

Rank p owns the experts `placement[p]` (E / P of them: its slice of the frozen int4 bank, its selected experts and
their LoRA factors); the router and the shared expert with its LoRA are replicated and every rank routes and combines
its own tokens. One call, on every rank at once:

  source  route its T tokens; plan, per destination rank, the tokens that have at least one expert there (one row
          per token and destination, however many of its K experts that rank owns), in token order, with the row's
          entries (local expert, k, routing weight); copy those rows into its exchange region
  owner   pull the rows addressed to it from every source's region over NVLink (one read per row), number their
          entries in (source, row, slot) order, build the expert dispatch of the entries (the stable counting sort of
          the single-GPU layer) and run its experts through the same fused GEMMs (smelb_moe_layer_fwd with an
          external dispatch); per received row, sum its entries' outputs times their weights in fp32 and publish
          that one partial row
  source  out[t] = the fp32 sum over the owners of t's partial rows, in rank order, plus the gated shared expert,
          which runs on the source's own tokens in the same GEMM launches as its share of the routed experts

Backward mirrors it with the upstream gradient: the owners form dY = g * w and d w = g . y per entry, run the expert
backward (dX and their LoRA gradients, which stay with the owner), and return one summed dX row per received row and
the d w of every entry. The shared expert's LoRA gradients are per-rank partial sums; `allreduce_shared_grads` adds
them (once per optimizer step).

The exchange lives in device memory the library allocates per rank and maps into the peers by CUDA IPC (EPGroup);
all synchronisation is device-side with bounded waits (csrc/ep.cu), so nothing synchronises with the host and a
training step stays capturable in a CUDA graph. Rounding differs from the single-GPU combine only in that each
owner's partial sum is rounded to bf16 before the source adds the partials.
"""
import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib
from .lora import ExpertsLoRA, LayerLoRA
from .moe import (_SAVE_PREACT, BF16Experts, Int4Experts, LayerExperts, _alloc_bwd, _alloc_fwd, _bf16, _Cfg, _fp32,
                  _LORA_NAMES, _set_routed, _set_shared, _struct, route)

SYNC = {"wait_done": 0, "publish": 1, "wait_ready": 2, "ack": 3}


# ------------------------------------------------------------------------------------------ placement
def expert_range(E: int, rank: int, world: int):
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    n = E // world
    return rank * n, (rank + 1) * n


def contiguous_placement(E: int, world: int):
    return [list(range(*expert_range(E, r, world))) for r in range(world)]


# The cost of an expert's routed rows on the owner's GEMMs, in row-equivalents: every row costs one, and a frozen
# int4 expert adds a fixed cost per 192-row token tile, the expansion of its whole weight tile into TMEM for that
# token tile. Fitted to the kernel times of a config-2 step (forward, recompute and backward: 959 us for the frozen
# experts' 16.4k rows over 244 experts, 300 us for the selected experts' 16.4k rows over 12): 18.3 ns per row for
# both kinds, 2.7 us (about 150 rows) per frozen expert token tile.
FROZEN_TILE_COST = 150.0
TOKEN_TILE_ROWS = 192


def expert_costs(ex, loads, frozen_tile: float = FROZEN_TILE_COST):
    """Per-expert cost of `loads` routed rows (row-equivalents) for balanced_placement; ex: LayerExperts."""
    sel = set(ex.sel_ids.tolist()) if ex.sel_ids is not None else set()
    out = []
    for e, c in enumerate(loads):
        c = float(c)
        tiles = math.ceil(c / TOKEN_TILE_ROWS) if c > 0 else 0
        out.append(c + (0.0 if e in sel else frozen_tile * tiles))
    return out


def balanced_placement(loads, world: int, cost=None):
    """E / world experts per rank with the routed cost balanced: the experts in decreasing cost (ties: smaller id)
    each go to the least-loaded rank that still has room (ties: smaller rank). Returns the sorted expert ids of every
    rank. `loads`: rows routed to each expert on a representative batch; `cost`: each expert's cost of those rows
    (expert_costs; default: the rows themselves)."""
    loads = [float(v) for v in loads]
    E = len(loads)
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    w = [float(cost[e]) for e in range(E)] if cost is not None else loads
    cap = E // world
    order = sorted(range(E), key=lambda e: (-w[e], e))
    tot = [0.0] * world
    out = [[] for _ in range(world)]
    for e in order:
        r = min((q for q in range(world) if len(out[q]) < cap), key=lambda q: (tot[q], q))
        out[r].append(e)
        tot[r] += w[e]
    return [sorted(v) for v in out]


class EPShard:
    """One rank's share of a layer: its experts (a LayerExperts over its local ids), its LoRA (the selected local
    experts' factors and the replicated shared LoRA), the placement and the device maps expert -> owner rank and
    expert -> local id."""

    def __init__(self, ex, lora, placement, rank, E):
        self.ex, self.lora, self.placement, self.rank, self.E = ex, lora, placement, rank, E
        self._dev = {}

    def maps(self, device):
        key = str(device)
        if key not in self._dev:
            owner = torch.empty(self.E, dtype=torch.int32)
            local = torch.empty(self.E, dtype=torch.int32)
            for r, ids in enumerate(self.placement):
                for j, e in enumerate(ids):
                    owner[e], local[e] = r, j
            meta = self.ex.meta(device)
            mask = torch.zeros(self.ex.E + 1, dtype=torch.uint8)  # + the sink expert of unused dispatch entries
            mask[:self.ex.E] = meta["sel_mask"].cpu()
            self._dev[key] = {"owner": owner.to(device), "local": local.to(device), "sel_mask_sink": mask.to(device)}
        return self._dev[key]


def shard_layer(ex: LayerExperts, lora_layer, rank: int, world: int, placement=None) -> EPShard:
    """Rank `rank`'s EPShard of a layer: the experts placement[rank] (default: contiguous ranges) as local ids 0..,
    their frozen-bank rows copied out of the bank, their selected experts and fresh Parameters with their LoRA
    factors; the shared LoRA is kept as it is (replicated)."""
    E = ex.E
    placement = placement or contiguous_placement(E, world)
    if len(placement) != world or sorted(e for p in placement for e in p) != list(range(E)):
        raise ValueError("placement must split all experts over the ranks")
    ids = list(placement[rank])
    idx = torch.tensor(ids, dtype=torch.long)
    fz = ex.frozen
    if isinstance(fz, Int4Experts):
        pick = lambda d: {k: v.index_select(0, idx.to(v.device)).contiguous() for k, v in d.items()}  # noqa: E731
        bank = Int4Experts(pick(fz.gu), pick(fz.dn), fz.dtype)
    elif isinstance(fz, BF16Experts):
        bank = BF16Experts(fz.gate_up.index_select(0, idx.to(fz.gate_up.device)).contiguous(),
                           fz.down.index_select(0, idx.to(fz.down.device)).contiguous())
    else:
        raise TypeError(f"shard_layer: unsupported bank {type(fz).__name__}")
    where = {e: j for j, e in enumerate(ids)}
    slots, loc_ids = [], []
    if ex.sel_ids is not None:
        for j, e in enumerate(ex.sel_ids.tolist()):
            if e in where:
                slots.append(j)
                loc_ids.append(where[e])
    if slots:
        ex_loc = LayerExperts(bank, loc_ids, ex.sel_gate_up[slots], ex.sel_down[slots], ex.group, ex.act)
    else:
        ex_loc = LayerExperts(bank, None, None, None, ex.group, ex.act)
    lora_loc = None
    if lora_layer is not None:
        le, le_loc = lora_layer.experts, None
        if le is not None and slots:
            H, I = le.A_gate.shape[2], le.B_gate.shape[1]
            le_loc = ExpertsLoRA(loc_ids, H, I, le.r, le.alpha).to(le.A_gate.device)
            with torch.no_grad():
                for n in _LORA_NAMES:
                    getattr(le_loc, n).copy_(getattr(le, n)[slots])
        lora_loc = LayerLoRA(le_loc, lora_layer.shared)
    return EPShard(ex_loc, lora_loc, placement, rank, E)


def allreduce_shared_grads(lora_layer, group=None):
    """Sum the replicated shared-expert LoRA gradients over the ranks (once per optimizer step)."""
    if lora_layer is None or lora_layer.shared is None:
        return
    for p in lora_layer.shared.parameters():
        if p.grad is not None:
            dist.all_reduce(p.grad, group=group)


# ------------------------------------------------------------------------------------------ exchange regions
class EPGroup:
    """The exchange regions of one expert-parallel group: this rank's (allocated by the library) and every peer's
    (mapped by CUDA IPC). `cap` is the most tokens a rank brings to one call, `K` the router's top-k. With one rank
    (or no process group) the exchange runs against the rank's own region. close() (after a barrier) unmaps and
    frees them."""

    def __init__(self, cap: int, H: int, K: int, group=None, device=None):
        self.group = group
        init = dist.is_available() and dist.is_initialized()
        self.P = dist.get_world_size(group) if init else 1
        self.rank = dist.get_rank(group) if init else 0
        self.cap, self.H, self.K = int(cap), int(H), int(K)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        nbytes = int(lib.smelb_ep_region_bytes(self.P, self.cap, self.K, self.H))
        if nbytes <= 0:
            raise _lib.SmelbError(f"EPGroup: unsupported shape P={self.P} cap={cap} K={K} H={H}")
        base = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        _lib.call("smelb_ep_region_alloc", nbytes, ctypes.byref(base), handle)
        self._own = base.value
        handles = [bytes(handle)]
        if self.P > 1:
            handles = [None] * self.P
            dist.all_gather_object(handles, bytes(handle), group=group)
        bases, self._opened = [], []
        for s in range(self.P):
            if s == self.rank:
                bases.append(self._own)
                continue
            h = (ctypes.c_char * 64).from_buffer_copy(handles[s])
            p = ctypes.c_void_p()
            _lib.call("smelb_ep_region_open", h, ctypes.byref(p))
            bases.append(p.value)
            self._opened.append(p.value)
        self._arr = (ctypes.c_void_p * self.P)(*bases)
        self.regions = ctypes.cast(self._arr, ctypes.c_void_p).value

    def sync(self, op: str, buffer: int):
        _lib.call("smelb_ep_sync", self.regions, self.P, self.rank, self.cap, self.K, self.H, SYNC[op], buffer,
                  _lib.stream_ptr(self.device))

    def close(self):
        for p in self._opened:
            _lib.call("smelb_ep_region_close", p)
        self._opened = []
        if self._own:
            _lib.call("smelb_ep_region_free", self._own)
            self._own = None


# ------------------------------------------------------------------------------------------ the routed part
def _i32(*s, dev):
    return torch.empty(*s, dtype=torch.int32, device=dev)


class _EPRoutedFn(torch.autograd.Function):
    """out = routed experts (partitioned over the group) + the gated shared expert. Inputs: x, topv, topi, shard, comm,
    cap_factor, shw (the shared expert's (gate_up, down, gate) weights), then the local selected experts' six LoRA
    parameters and the shared expert's six (or None)."""

    @staticmethod
    def forward(ctx, x, topv, topi, shard, comm, cap_factor, shw, *lora_params):
        dev = x.device
        T, H = x.shape
        K = topi.shape[1]
        P, r, cap = comm.P, comm.rank, comm.cap
        if T > cap or H != comm.H or K != comm.K:
            raise _lib.SmelbError(f"moe_forward_ep: T={T} H={H} K={K} against the group's cap={cap} H={comm.H} "
                                  f"K={comm.K}")
        maps = shard.maps(dev)
        ex = shard.ex
        E_loc = ex.E
        cap_e = int(math.ceil(cap_factor * cap * K))
        st = _lib.stream_ptr(dev)
        reg = comm.regions
        topi = topi.contiguous()
        f32 = topv.dtype == torch.float32
        topv = topv.contiguous()
        # ---- source: plan and publish the token rows (buffer 0)
        pos, slot_j, tok_of = _i32(T, P, dev=dev), _i32(T, K, dev=dev), _i32(P, cap, dev=dev)
        comm.sync("wait_done", 0)
        _lib.call("smelb_ep_plan", _lib.ptr(topi), _lib.ptr(topv), 1 if f32 else 0, T, K, _lib.ptr(maps["owner"]),
                  _lib.ptr(maps["local"]), reg, P, r, cap, H, _lib.ptr(pos), _lib.ptr(slot_j), _lib.ptr(tok_of), st)
        _lib.call("smelb_ep_pack_rows", _lib.ptr(x), H, _lib.ptr(tok_of), reg, P, r, cap, K, 0, st)
        comm.sync("publish", 0)
        # ---- owner: pull, number the entries, dispatch them to the local experts
        comm.sync("wait_ready", 0)
        entry_e = torch.empty(cap_e, dtype=torch.int64, device=dev)
        entry_row, entry_w = _i32(cap_e, dev=dev), torch.empty(cap_e, dtype=torch.float32, device=dev)
        row_beg, row_m, rc, n_tot = _i32(P * cap, dev=dev), _i32(P * cap, dev=dev), _i32(P, dev=dev), _i32(1, dev=dev)
        _lib.call("smelb_ep_recv_plan", reg, P, r, cap, K, H, cap_e, E_loc, _lib.ptr(entry_e), _lib.ptr(entry_row),
                  _lib.ptr(entry_w), _lib.ptr(row_beg), _lib.ptr(row_m), _lib.ptr(rc), _lib.ptr(n_tot), st)
        x_loc = torch.empty(P * cap, H, dtype=torch.bfloat16, device=dev)
        _lib.call("smelb_ep_pull_rows", reg, P, r, cap, K, H, 0, _lib.ptr(x_loc), st)
        comm.sync("ack", 0)
        lora_ex = shard.lora.experts if shard.lora is not None else None
        lora_sh = shard.lora.shared if shard.lora is not None else None
        # the owner's experts on its received entries (cap_e dispatch "tokens" of weight 1) and the shared expert on
        # this rank's T tokens, one layer call: the buffers of each from its own description, then one struct
        cfg = _Cfg(0, torch.empty(cap_e, H, device="meta"), 1, E_loc, ex.act)
        _set_routed(cfg, ex, lora_ex, dev)
        cfg_sh = _Cfg(0, x, 0, 0)
        _set_shared(cfg_sh, shw[0], shw[1], lora_sh, shw[2])
        save = any(ctx.needs_input_grad)
        t = dict(cfg.t)
        t.update(_alloc_fwd(cfg, dev, save))
        t.pop("out")  # the owner's outputs stay in dispatch order (y)
        t.update(cfg_sh.t)
        t.update({k: v for k, v in _alloc_fwd(cfg_sh, dev, save).items() if k != "out"})
        R = cfg.max_rows
        cfg.flags |= cfg_sh.flags | _lib.F_EXT_DISPATCH
        cfg.T, cfg.S, cfg.r_sh, cfg.s_sh, cfg.act_sh = T, cfg_sh.S, cfg_sh.r_sh, cfg_sh.s_sh, cfg_sh.act_sh
        if save:
            cfg.flags |= _lib.F_SAVE
            if not _SAVE_PREACT[0]:
                cfg.flags |= _lib.F_RECOMPUTE
        t["x"] = x
        lp = [_fp32(p) for p in lora_params]
        for i, name in enumerate(_LORA_NAMES):
            t[name], t["sh" + name] = lp[i], lp[6 + i]
        t.update(counts=_i32(E_loc + 1, dev=dev), gcounts=_i32(E_loc + 1, dev=dev), offsets=_i32(E_loc + 1, dev=dev))
        ws = _i32(148 * (E_loc + 1), dev=dev)
        _lib.call("smelb_dispatch_plan_ws", _lib.ptr(entry_e), cap_e, 1, E_loc + 1, _lib.ptr(maps["sel_mask_sink"]),
                  64, _lib.ptr(t["counts"]), _lib.ptr(t["gcounts"]), _lib.ptr(t["offsets"]), _lib.ptr(t["row_of"]),
                  _lib.ptr(t["src_of"]), _lib.ptr(t["order"]), _lib.ptr(t["total"]), _lib.ptr(ws), ws.numel(), st)
        _lib.call("smelb_ep_gather", _lib.ptr(x_loc), _lib.ptr(entry_row), _lib.ptr(t["src_of"]),
                  _lib.ptr(t["offsets"]), E_loc, H, R, _lib.ptr(t["xs"]), st)
        L = _struct(cfg, t)
        _lib.call("smelb_moe_layer_fwd", ctypes.byref(L))
        # ---- owner: one partial row per received row (buffer 1)
        comm.sync("wait_done", 1)
        _lib.call("smelb_ep_return", _lib.ptr(t["y"]), _lib.ptr(t["row_of"]), _lib.ptr(entry_w), None,
                  _lib.ptr(row_beg), _lib.ptr(row_m), _lib.ptr(rc), reg, P, r, cap, K, H, 0, st)
        comm.sync("publish", 1)
        # ---- source: add the partial rows of every owner and the shared expert
        comm.sync("wait_ready", 1)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        _lib.call("smelb_ep_collect", reg, P, r, cap, K, H, T, _lib.ptr(pos), _lib.ptr(t["sh_y"]),
                  _lib.ptr(t.get("sgate_logit")), None, None, 0, None, None, None, None, 0, _lib.ptr(out), st)
        comm.sync("ack", 1)
        if save:
            ctx.save_for_backward(topi, pos, slot_j, tok_of, entry_row, entry_w, row_beg, row_m, rc)
            ctx.t, ctx.cfg, ctx.shard, ctx.comm = t, cfg, shard, comm
            ctx.meta = (T, H, K, E_loc, R, f32, [None if p is None else p.dtype for p in lora_params])
        return out

    @staticmethod
    def backward(ctx, g):
        topi, pos, slot_j, tok_of, entry_row, entry_w, row_beg, row_m, rc = ctx.saved_tensors
        t, cfg, shard, comm = dict(ctx.t), ctx.cfg, ctx.shard, ctx.comm
        T, H, K, E_loc, R, f32, dtypes = ctx.meta
        P, r, cap = comm.P, comm.rank, comm.cap
        dev = g.device
        st = _lib.stream_ptr(dev)
        reg = comm.regions
        g = g.to(torch.bfloat16).contiguous()
        maps = shard.maps(dev)
        # ---- source: the gradient rows of the same token rows (buffer 2)
        comm.sync("wait_done", 2)
        _lib.call("smelb_ep_pack_rows", _lib.ptr(g), H, _lib.ptr(tok_of), reg, P, r, cap, K, 2, st)
        comm.sync("publish", 2)
        # ---- owner: pull them, dY and d w per entry, the expert backward
        comm.sync("wait_ready", 2)
        g_loc = torch.empty(P * cap, H, dtype=torch.bfloat16, device=dev)
        _lib.call("smelb_ep_pull_rows", reg, P, r, cap, K, H, 2, _lib.ptr(g_loc), st)
        comm.sync("ack", 2)
        b = _alloc_bwd(cfg, dev)
        t.update(b)
        t["g"] = g  # the shared expert's upstream gradient (this rank's tokens)
        entry_dw = torch.zeros(entry_w.shape, dtype=torch.float32, device=dev)
        _lib.call("smelb_ep_dy", _lib.ptr(g_loc), _lib.ptr(entry_row), _lib.ptr(entry_w), _lib.ptr(t["src_of"]),
                  _lib.ptr(t["offsets"]), E_loc, H, R, _lib.ptr(t["y"]), _lib.ptr(t["dy"]), _lib.ptr(entry_dw), st)
        L = _struct(cfg, t)
        _lib.call("smelb_moe_layer_bwd", ctypes.byref(L))
        # ---- owner: summed dX per received row and d w per entry (buffer 3)
        comm.sync("wait_done", 3)
        _lib.call("smelb_ep_return", _lib.ptr(t["dxs"]), _lib.ptr(t["row_of"]), None, _lib.ptr(entry_dw),
                  _lib.ptr(row_beg), _lib.ptr(row_m), _lib.ptr(rc), reg, P, r, cap, K, H, 1, st)
        comm.sync("publish", 3)
        # ---- source: dX of its tokens and d topv
        comm.sync("wait_ready", 3)
        dx = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        dtopv = torch.empty(T, K, dtype=torch.float32 if f32 else torch.bfloat16, device=dev)
        _lib.call("smelb_ep_collect", reg, P, r, cap, K, H, T, _lib.ptr(pos), _lib.ptr(t["sh_dx"]), None,
                  _lib.ptr(t.get("dgl")), _lib.ptr(t.get("w_sgate")) if "dgl" in t else None, 1, _lib.ptr(topi),
                  _lib.ptr(maps["owner"]), _lib.ptr(slot_j), _lib.ptr(dtopv), 1 if f32 else 0, _lib.ptr(dx), st)
        comm.sync("ack", 3)
        grads = [b.get("g" + n) for n in _LORA_NAMES] + [b.get("gsh" + n) for n in _LORA_NAMES]
        grads = [None if (gr is None or dt is None) else gr.to(dt) for gr, dt in zip(grads, dtypes)]
        return (dx, dtopv, None, None, None, None, None, *grads)


def moe_forward_ep(x2d, W, shard: EPShard, top_k: int, comm: EPGroup, stats=None, cap_factor: float = 2.0):
    """moe_forward (moe.py:255-263) with the routed experts partitioned over `comm`'s ranks.

    x2d: this rank's tokens [T, H] bf16 (T <= comm.cap); W: the replicated router / shared-expert tensors; shard:
    this rank's EPShard. Every rank of the group must make the same sequence of calls. cap_factor bounds the
    dispatch entries an owner can take (cap_factor * cap * top_k); more record a device status code. Returns this
    rank's [T, H] output, differentiable w.r.t. x2d, the local selected experts' LoRA parameters and the shared LoRA
    parameters."""
    x2d = _bf16(x2d, "moe_forward_ep: x")
    probs, topv, topi = route(x2d, W["mlp.gate.weight"], top_k)
    if stats is not None:
        stats(probs, topv, topi)
    pre = "mlp.shared_expert."
    gu = W.get(pre + "gate_up_proj.weight")
    if gu is None:
        gu = torch.cat((W[pre + "gate_proj.weight"], W[pre + "up_proj.weight"]))
    shw = (gu, W[pre + "down_proj.weight"], W["mlp.shared_expert_gate.weight"])
    lex = shard.lora.experts if shard.lora is not None else None
    lsh = shard.lora.shared if shard.lora is not None else None
    params = ([getattr(lex, n) for n in _LORA_NAMES] if lex is not None else [None] * 6) + \
             ([getattr(lsh, n) for n in _LORA_NAMES] if lsh is not None else [None] * 6)
    return _EPRoutedFn.apply(x2d, topv, topi, shard, comm, float(cap_factor), shw, *params)
