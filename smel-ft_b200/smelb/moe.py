"""The MoE expert layer of SMEL FT (smel/moe.py:1-263) on B200: same classes, functions and autograd behaviour,
computed by the fused sm_100a kernels of libsmelb.

  route            router GEMM -> fp32 softmax -> top-k (ties to the smaller expert id) -> renorm (moe.py:162-167)
  routed_experts   stable counting-sort dispatch -> frozen int4 experts (dequant fused into the GEMM producer) and
                   selected bf16 experts with LoRA in the GEMM K-extension -> fp32 weighted combine (moe.py:214-252)
  shared_mlp       gated MLP with LoRA and the sigmoid shared-expert gate (moe.py:183-201)
  moe_forward      all of the above as one forward call and one backward call (moe.py:255-263)
  FrozenExpertsFn  frozen experts alone (int4 or bf16 bank), dX only in backward (moe.py:110-143)

Activation memory: by default the forward under autograd keeps the gate/up pre-activations h [rows, 2I] (and the
shared expert's), so the backward skips one gate/up GEMM. set_save_preactivations(False) restores the reference's
contract (FrozenExpertsFn saves only xs, moe.py:1-5 and :123): the backward then recomputes h first.

Activations are bf16 on CUDA. There is no CPU path: CPU tensors raise SmelbError.
"""
import ctypes

import torch

from . import _lib
from .quant import dequant_int4, pack_sz, quantize_int4

_LORA_NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")
_W64 = 64  # width of the LoRA token-side buffers (2r <= 64)
_SAVE_PREACT = [True]


def set_save_preactivations(flag: bool):
    """Keep the gate/up pre-activations from the forward for the backward (True, the default: one GEMM less per
    backward, R x 2I bf16 more activation memory per layer call) or recompute them in the backward from the saved
    inputs (False: the reference's activation memory)."""
    _SAVE_PREACT[0] = bool(flag)


def save_preactivations() -> bool:
    return _SAVE_PREACT[0]


# ==================================================================================================== weight banks
class BF16Experts:
    """Frozen experts as fused bf16 tensors: gate_up [E, 2I, H], down [E, H, I] (moe.py:18-32)."""

    def __init__(self, gate_up: torch.Tensor, down: torch.Tensor):
        self.gate_up, self.down = gate_up, down
        self.num_experts = gate_up.shape[0]

    def weights(self, e0: int, e1: int):
        return self.gate_up[e0:e1], self.down[e0:e1]

    def tensors(self):
        return {"gate_up": self.gate_up, "down": self.down}

    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in self.tensors().values())

    def kernel_operands(self):
        if self.gate_up.dtype != torch.bfloat16 or self.down.dtype != torch.bfloat16:
            raise _lib.SmelbError("BF16Experts: the fused kernels take bf16 banks")
        return {"fz_gu": self.gate_up.contiguous(), "fz_dn": self.down.contiguous()}


class Int4Experts:
    """Frozen experts in group-wise int4 (moe.py:35-55). gu / dn are dicts with q (uint8 [E, N, K/2]),
    scale and zero (bf16 [E, N, K/64]). The fused GEMMs read q directly and a transposed copy of the
    (scale, zero) pairs built once on first use."""

    def __init__(self, gu: dict, dn: dict, dtype=torch.bfloat16):
        self.gu, self.dn, self.dtype = gu, dn, dtype
        self.num_experts = gu["q"].shape[0]
        self._sz = None

    @classmethod
    def from_bf16(cls, gate_up, down, group=64):
        return cls(quantize_int4(gate_up, group), quantize_int4(down, group), dtype=gate_up.dtype)

    def weights(self, e0: int, e1: int):
        gu = dequant_int4(self.gu["q"][e0:e1], self.gu["scale"][e0:e1], self.gu["zero"][e0:e1], self.dtype)
        dn = dequant_int4(self.dn["q"][e0:e1], self.dn["scale"][e0:e1], self.dn["zero"][e0:e1], self.dtype)
        return gu, dn

    def tensors(self):
        return {f"gate_up.{k}": v for k, v in self.gu.items()} | {f"down.{k}": v for k, v in self.dn.items()}

    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in self.tensors().values())

    def kernel_operands(self):
        for name, d in (("gate_up", self.gu), ("down", self.dn)):
            k = d["q"].shape[-1] * 2
            if d["scale"].shape[-1] * 64 != k:
                raise _lib.SmelbError(f"Int4Experts.{name}: the fused kernels take group-64 banks "
                                      f"(K={k}, {d['scale'].shape[-1]} groups)")
        if self._sz is None:
            self._sz = (pack_sz(self.gu["scale"], self.gu["zero"]), pack_sz(self.dn["scale"], self.dn["zero"]))
        return {"gu_q": self.gu["q"].contiguous(), "gu_sz": self._sz[0], "dn_q": self.dn["q"].contiguous(),
                "dn_sz": self._sz[1]}


class LayerExperts:
    """Routed experts of one layer: the frozen bank for all E experts plus optional trainable bf16 copies of the
    selected experts, whose frozen-bank copy is then ignored (moe.py:146-159)."""

    def __init__(self, frozen, sel_ids=None, sel_gate_up=None, sel_down=None, group: int = 32, act: str = "silu"):
        self.frozen = frozen
        self.E = frozen.num_experts
        self.group = group  # expert-group size of the reference's dequant loop; the fused kernels do not need it
        self.act = act
        self.sel_ids = None if sel_ids is None else torch.as_tensor(sel_ids, dtype=torch.long)
        self.sel_gate_up, self.sel_down = sel_gate_up, sel_down
        self._slot = {}
        if self.sel_ids is not None:
            self._slot = {int(e): j for j, e in enumerate(self.sel_ids.tolist())}
        self._meta = {}

    def meta(self, device):
        """Device-side index tensors of the selection (cached per device)."""
        key = str(device)
        if key not in self._meta:
            sel = self.sel_ids.tolist() if (self.sel_ids is not None and len(self._slot)) else []
            frozen = [e for e in range(self.E) if e not in set(sel)]
            mask = torch.zeros(self.E, dtype=torch.uint8)
            mask[sel] = 1
            self._meta[key] = {
                "frozen_ids": torch.tensor(frozen, dtype=torch.int32).to(device),
                "sel_ids": torch.tensor(sel, dtype=torch.int32).to(device),
                "sel_slots": torch.arange(len(sel), dtype=torch.int32).to(device),
                "sel_mask": mask.to(device),
                "n_sel": len(sel),
            }
        return self._meta[key]


# ==================================================================================================== the fused call
class _Cfg:
    """Non-tensor description of one layer call (which sub-paths, shapes, weights)."""

    def __init__(self, flags, x, top_k=0, E=0, act="silu"):
        self.flags = flags
        self.T, self.H = x.shape
        self.K, self.E = top_k, E
        self.I = self.S = self.n_sel = self.r_sel = self.r_sh = 0
        self.s_sel = self.s_sh = 0.0
        if act not in _lib.ACT:
            raise ValueError(f"unknown activation {act}")
        self.act = act
        self.act_sh = act
        self.t = {}  # weight tensors by struct field name
        self.lora_dtypes = [None] * 12
        self.topv_dtype = torch.bfloat16


def _bf16(t, what):
    if t is None:
        return None
    if not t.is_cuda:
        raise _lib.SmelbError(f"{what}: smelb runs on CUDA tensors only")
    if t.dtype != torch.bfloat16:
        raise _lib.SmelbError(f"{what}: expected bf16, got {t.dtype}")
    return t.contiguous()


def _lora_params(lora):
    if lora is None:
        return [None] * 6
    return [getattr(lora, n) for n in _LORA_NAMES]


def _fp32(p):
    return None if p is None else p.detach().float().contiguous()


def _set_routed(cfg, ex: LayerExperts, lora_ex, dev):
    cfg.flags |= _lib.F_ROUTED
    bank = ex.frozen
    ops = bank.kernel_operands()
    cfg.t.update(ops)
    if "gu_q" in ops:
        cfg.I = ops["dn_q"].shape[-1] * 2
    else:
        cfg.I = ops["fz_dn"].shape[-1]
    meta = ex.meta(dev)
    cfg.t.update({k: meta[k] for k in ("frozen_ids", "sel_ids", "sel_slots", "sel_mask")})
    cfg.n_sel = meta["n_sel"]
    cfg.act = ex.act
    if cfg.n_sel:
        cfg.t["sel_gu"] = _bf16(ex.sel_gate_up, "sel_gate_up")
        cfg.t["sel_dn"] = _bf16(ex.sel_down, "sel_down")
        if lora_ex is not None:
            cfg.r_sel, cfg.s_sel = lora_ex.r, float(lora_ex.scale)
    if cfg.E and cfg.E != bank.num_experts:
        raise _lib.SmelbError(f"router has {cfg.E} experts, bank has {bank.num_experts}")
    cfg.E = bank.num_experts


def _set_shared(cfg, w_gate_up, w_down, lora_sh, w_sgate=None):
    cfg.flags |= _lib.F_SHARED
    cfg.t["sh_gu"] = _bf16(w_gate_up, "shared gate_up")
    cfg.t["sh_dn"] = _bf16(w_down, "shared down")
    cfg.S = w_down.shape[1]
    if lora_sh is not None:
        cfg.r_sh, cfg.s_sh = lora_sh.r, float(lora_sh.scale)
    if w_sgate is not None:
        cfg.flags |= _lib.F_SHARED_GATE
        cfg.t["w_sgate"] = _bf16(w_sgate, "shared_expert_gate")


def _alloc_fwd(cfg, dev, save):
    T, H, E, K, I, S, n, r, rh = cfg.T, cfg.H, cfg.E, cfg.K, cfg.I, cfg.S, cfg.n_sel, cfg.r_sel, cfg.r_sh
    f = cfg.flags
    b = {"out": torch.empty(T, H, dtype=torch.bfloat16, device=dev),
         "tok_count": torch.full((1,), T, dtype=torch.int32, device=dev)}
    e = lambda *s, dtype=torch.bfloat16: torch.empty(*s, dtype=dtype, device=dev)  # noqa: E731
    if f & _lib.F_ROUTER:
        b.update(logits=e(T, E), probs=e(T, E, dtype=torch.float32), topv=e(T, K, dtype=cfg.topv_dtype),
                 topi=e(T, K, dtype=torch.int64))
    if f & _lib.F_SHARED_GATE:
        b["sgate_logit"] = e(T)
    if f & _lib.F_ROUTED:
        R = T * K + n * 64
        cfg.max_rows = R
        b.update(counts=e(E, dtype=torch.int32), gcounts=e(E, dtype=torch.int32), offsets=e(E, dtype=torch.int32),
                 row_of=e(T * K, dtype=torch.int32), src_of=e(R, dtype=torch.int32), total=e(1, dtype=torch.int32),
                 order=e(T * K, dtype=torch.int64), xs=e(R, H), a=e(R, I), y=e(R, H),
                 split_counts=e(2 * (E + 1), dtype=torch.int32))
        if save and _SAVE_PREACT[0]:
            b["h"] = e(R, 2 * I)
        if n and r:
            # the 64-wide LoRA blocks: the GEMMs write every row of the selected segments, padding columns as zeros
            b.update(xa=e(R, _W64), z=e(R, _W64), p_xa_w=e(n, 2 * r, H), p_gu_ext=e(n, 2 * I, _W64),
                     p_z_w=e(n, r, I), p_dn_ext=e(n, H, _W64))
    else:
        cfg.max_rows = 0
    if f & _lib.F_SHARED:
        b.update(sh_a=e(T, S), sh_y=e(T, H))
        if save and _SAVE_PREACT[0]:
            b["sh_h"] = e(T, 2 * S)
        if rh:
            b.update(sh_xa=e(T, _W64), sh_z=e(T, _W64), sp_xa_w=e(1, 2 * rh, H), sp_gu_ext=e(1, 2 * S, _W64),
                     sp_z_w=e(1, rh, S), sp_dn_ext=e(1, H, _W64))
    return b


def _alloc_bwd(cfg, dev):
    T, H, E, K, I, S, n, r, rh = cfg.T, cfg.H, cfg.E, cfg.K, cfg.I, cfg.S, cfg.n_sel, cfg.r_sel, cfg.r_sh
    f = cfg.flags
    e = lambda *s, dtype=torch.bfloat16: torch.empty(*s, dtype=dtype, device=dev)  # noqa: E731
    z = lambda *s, dtype=torch.bfloat16: torch.zeros(*s, dtype=dtype, device=dev)  # noqa: E731
    b = {"dx": e(T, H)}
    if f & _lib.F_RECOMPUTE:  # the forward kept no pre-activations: the backward recomputes them here
        if f & _lib.F_ROUTED:
            b["h"] = e(cfg.max_rows, 2 * I)
        if f & _lib.F_SHARED:
            b["sh_h"] = e(T, 2 * S)
    if f & _lib.F_ROUTED:
        R = cfg.max_rows
        b.update(dy=e(R, H), dh=e(R, 2 * I), dxs=e(R, H), dtopv=e(T, K, dtype=cfg.topv_dtype))
        if n and r:
            b.update(dz=e(R, _W64), dxa=e(R, _W64), p_dz_w=e(n, r, H), p_da_ext=e(n, I, _W64),
                     p_dxa_w=e(n, 2 * r, 2 * I), p_dx_ext=e(n, H, _W64))
            for name, shp in zip(_LORA_NAMES, ((n, r, H), (n, I, r), (n, r, H), (n, I, r), (n, r, I), (n, H, r))):
                b["g" + name] = e(*shp, dtype=torch.float32)
    if f & _lib.F_ROUTER:
        Ep = (E + 63) // 64 * 64  # padding columns (E % 64 != 0) must read as zero; the router backward writes the rest
        b.update(dlogits=(e if Ep == E else z)(T, Ep), dx_router=e(T, H))
        if "dtopv" not in b:
            b["dtopv"] = e(T, K, dtype=cfg.topv_dtype)
    if f & _lib.F_SHARED:
        b.update(sh_dh=e(T, 2 * S), sh_dx=e(T, H))
        if f & _lib.F_SHARED_GATE:
            b.update(sh_dy=e(T, H), dgl=e(T, dtype=torch.float32))
        if rh:
            b.update(sh_dz=e(T, _W64), sh_dxa=e(T, _W64), sp_dz_w=e(1, rh, H), sp_da_ext=e(1, S, _W64),
                     sp_dxa_w=e(1, 2 * rh, 2 * S), sp_dx_ext=e(1, H, _W64))
            for name, shp in zip(_LORA_NAMES, ((rh, H), (S, rh), (rh, H), (S, rh), (rh, S), (H, rh))):
                b["gsh" + name] = e(*shp, dtype=torch.float32)
    return b


def _struct(cfg, tensors: dict):
    L = _lib.MoELayerStruct()
    L.T, L.H, L.E, L.K, L.I, L.S = cfg.T, cfg.H, cfg.E, cfg.K, cfg.I, cfg.S
    L.n_sel, L.r_sel, L.r_sh, L.s_sel, L.s_sh = cfg.n_sel, cfg.r_sel, cfg.r_sh, cfg.s_sel, cfg.s_sh
    L.act, L.act_sh, L.flags, L.max_rows = _lib.ACT[cfg.act], _lib.ACT[cfg.act_sh], cfg.flags, cfg.max_rows
    L.stream = _lib.stream_ptr()
    for k, v in tensors.items():
        if v is not None and hasattr(L, k):
            setattr(L, k, _lib.ptr(v))
    return L


class _MoELayerFn(torch.autograd.Function):
    """One forward and one backward launch sequence for any combination of router / routed / shared sub-paths.
    Inputs: x, topv_in (routing given), cfg, then the 6 expert and 6 shared LoRA parameters (or None)."""

    @staticmethod
    def forward(ctx, x, topv_in, cfg, *params):
        dev = x.device
        save = any(ctx.needs_input_grad)
        cfg.flags &= ~(_lib.F_SAVE | _lib.F_RECOMPUTE)
        if save:
            cfg.flags |= _lib.F_SAVE
            if not _SAVE_PREACT[0] and cfg.flags & (_lib.F_ROUTED | _lib.F_SHARED):
                cfg.flags |= _lib.F_RECOMPUTE
        lp = [_fp32(p) for p in params]
        t = dict(cfg.t)
        t["x"] = x
        if topv_in is not None:
            t["topv_in"] = topv_in.contiguous()
        for i, name in enumerate(_LORA_NAMES):
            t[name], t["sh" + name] = lp[i], lp[6 + i]
        t.update(_alloc_fwd(cfg, dev, save))
        L = _struct(cfg, t)
        _lib.call("smelb_moe_layer_fwd", ctypes.byref(L))
        outs = (t["out"], t.get("probs", x.new_empty(0)), t.get("topv", x.new_empty(0)),
                t.get("topi", x.new_empty(0, dtype=torch.long)))
        # The function's own outputs are saved through save_for_backward and kept out of ctx: a plain reference
        # from ctx to an output forms a cycle through the output's grad_fn, which keeps the whole step's buffers
        # alive until Python's cycle collector runs (the caching allocator then grows and calls the driver).
        ctx.out_keys = [k for k in ("probs", "topv", "topi") if k in t]
        ctx.save_for_backward(*[t[k] for k in ctx.out_keys])
        ctx.out_shape = tuple(t["out"].shape)
        ctx.t = {k: v for k, v in t.items() if k not in ("out", "probs", "topv", "topi")}
        ctx.cfg, ctx.dtypes = cfg, [None if p is None else p.dtype for p in params]
        ctx.has_topv_in = topv_in is not None
        ctx.mark_non_differentiable(outs[3])
        return outs

    @staticmethod
    def backward(ctx, g_out, g_probs, g_topv, g_topi):
        cfg, t = ctx.cfg, dict(ctx.t)
        t.update(zip(ctx.out_keys, ctx.saved_tensors))
        dev = t["x"].device
        b = _alloc_bwd(cfg, dev)
        t.update(b)
        if g_out is None:
            g_out = torch.zeros(ctx.out_shape, dtype=torch.bfloat16, device=dev)
        t["g"] = g_out.to(torch.bfloat16).contiguous()
        if cfg.flags & _lib.F_ROUTER:
            if g_probs is not None and g_probs.numel():
                t["dprobs"] = g_probs.float().contiguous()
            if not (cfg.flags & _lib.F_ROUTED):
                b["dtopv"].copy_(g_topv if g_topv is not None else torch.zeros_like(b["dtopv"]))
        L = _struct(cfg, t)
        _lib.call("smelb_moe_layer_bwd", ctypes.byref(L))
        grads = []
        for i, name in enumerate(_LORA_NAMES):
            grads.append(b.get("g" + name))
        for i, name in enumerate(_LORA_NAMES):
            grads.append(b.get("gsh" + name))
        grads = [None if (gr is None or dt is None) else gr.to(dt) for gr, dt in zip(grads, ctx.dtypes)]
        d_topv = b.get("dtopv") if ctx.has_topv_in else None
        return (b["dx"], d_topv, None, *grads)


def _apply(cfg, x, topv_in=None, lora_ex=None, lora_sh=None):
    params = _lora_params(lora_ex) + _lora_params(lora_sh)
    return _MoELayerFn.apply(x, topv_in, cfg, *params)


# ==================================================================================================== public API
def route(x2d, gate_w, top_k):
    """(probs fp32 [N, E], topv [N, K] in the logits dtype, topi int64 [N, K]) (moe.py:162-167)."""
    x2d = _bf16(x2d, "route: x")
    cfg = _Cfg(_lib.F_ROUTER, x2d, top_k, gate_w.shape[0])
    cfg.t["w_router"] = _bf16(gate_w, "route: gate weight")
    _, probs, topv, topi = _apply(cfg, x2d)
    return probs, topv, topi


def route_gemma4(h, W, top_k, eps):
    """Gemma 4 router on the residual stream (moe.py:170-180): the weightless RMSNorm of h times router.scale times
    H^-0.5 (bf16 steps), router.proj logits, fp32 softmax, top-k renormalised in fp32 and multiplied by
    router.per_expert_scale of the chosen experts. Returns (probs fp32 [N, E], topv fp32 [N, K], topi int64 [N, K]);
    differentiable w.r.t. h through topv and probs."""
    from . import norm
    h = _bf16(h, "route_gemma4: h")
    x = norm.router_prologue_gemma4(h, W["router.scale"], eps)
    proj = W["router.proj.weight"]
    cfg = _Cfg(_lib.F_ROUTER | _lib.F_TOPV_FP32, x, top_k, proj.shape[0])
    cfg.topv_dtype = torch.float32
    cfg.t["w_router"] = _bf16(proj, "route_gemma4: router.proj.weight")
    cfg.t["per_expert_scale"] = _bf16(W["router.per_expert_scale"], "route_gemma4: router.per_expert_scale")
    _, probs, topv, topi = _apply(cfg, x)
    return probs, topv, topi


def routed_experts(x2d, topv, topi, ex: LayerExperts, lora=None):
    """Weighted sum of the routed experts for every token; differentiable w.r.t. x2d, topv and the LoRA parameters
    (moe.py:214-252)."""
    x2d = _bf16(x2d, "routed_experts: x")
    cfg = _Cfg(0, x2d, topi.shape[1], ex.E, ex.act)
    cfg.topv_dtype = topv.dtype
    if topv.dtype == torch.float32:
        cfg.flags |= _lib.F_TOPV_FP32
    elif topv.dtype != torch.bfloat16:
        raise _lib.SmelbError(f"routed_experts: topv dtype {topv.dtype} (bf16 or fp32)")
    _set_routed(cfg, ex, lora, x2d.device)
    cfg.t["topi_in"] = topi.contiguous()
    out = _apply(cfg, x2d, topv, lora_ex=lora)[0]
    return out


def mlp_lora(x, w_gate, w_up, w_down, lora, act_name="silu", w_gate_up=None):
    """down(act(gate(x)) * up(x)) with optional LoRA on all three projections (moe.py:183-194)."""
    shape = x.shape
    x2 = _bf16(x.reshape(-1, shape[-1]), "mlp_lora: x")
    cfg = _Cfg(0, x2, act=act_name)
    cfg.act_sh = act_name
    if w_gate_up is None:
        w_gate_up = torch.cat((w_gate, w_up))
    _set_shared(cfg, w_gate_up, w_down, lora)
    out = _apply(cfg, x2, lora_sh=lora)[0]
    return out.reshape(*shape[:-1], out.shape[-1])


def shared_mlp(x, W, lora):
    """Shared expert with LoRA times sigmoid(shared_expert_gate(x)) (moe.py:197-201)."""
    pre = "mlp.shared_expert."
    x = _bf16(x, "shared_mlp: x")
    cfg = _Cfg(0, x)  # the shared expert is SiLU (moe.py:197-201 calls mlp_lora with its default)
    gu = W.get(pre + "gate_up_proj.weight")
    if gu is None:
        gu = torch.cat((W[pre + "gate_proj.weight"], W[pre + "up_proj.weight"]))
    _set_shared(cfg, gu, W[pre + "down_proj.weight"], lora, W["mlp.shared_expert_gate.weight"])
    return _apply(cfg, x, lora_sh=lora)[0]


def moe_forward(x2d, W, ex: LayerExperts, top_k: int, lora_layer=None, stats=None):
    """route -> routed_experts + shared_mlp in one fused forward and one fused backward (moe.py:255-263).
    x2d [N, H] bf16 (already post-attention-normed); W holds the router and shared-expert tensors of the layer;
    stats(probs, topv, topi) is called once per call."""
    x2d = _bf16(x2d, "moe_forward: x")
    lora_ex = lora_layer.experts if lora_layer is not None else None
    lora_sh = lora_layer.shared if lora_layer is not None else None
    cfg = _Cfg(_lib.F_ROUTER, x2d, top_k, W["mlp.gate.weight"].shape[0], ex.act)
    cfg.t["w_router"] = _bf16(W["mlp.gate.weight"], "router weight")
    _set_routed(cfg, ex, lora_ex, x2d.device)
    cfg.act_sh = "silu"  # shared_mlp uses mlp_lora's default activation (moe.py:197-201)
    pre = "mlp.shared_expert."
    gu = W.get(pre + "gate_up_proj.weight")
    if gu is None:
        gu = torch.cat((W[pre + "gate_proj.weight"], W[pre + "up_proj.weight"]))
    _set_shared(cfg, gu, W[pre + "down_proj.weight"], lora_sh, W["mlp.shared_expert_gate.weight"])
    out, probs, topv, topi = _apply(cfg, x2d, lora_ex=lora_ex, lora_sh=lora_sh)
    if stats is not None:
        stats(probs, topv, topi)
    return out


def moe_block_gemma4(h, xm, W, ex: LayerExperts, top_k: int, eps: float, act="gelu_tanh", lora_layer=None,
                     stats=None):
    """The Gemma 4 MoE block of smel/layer_runner.py:249-261 after the attention residual: the dense MLP (with the
    layer's "shared" LoRA) on xm and the routed experts on the pre-FFN-2 norm of h run in parallel, each with its
    post norm, and  h + rmsnorm(m + e)  scaled by layer_scalar. Norms are Gemma's x * rstd * w."""
    from . import norm
    lora_sh = lora_layer.shared if lora_layer is not None else None
    lora_ex = lora_layer.experts if lora_layer is not None else None
    m = mlp_lora(xm, W["mlp.gate_proj.weight"], W["mlp.up_proj.weight"], W["mlp.down_proj.weight"], lora_sh, act,
                 W.get("mlp.gate_up_proj.weight"))
    m = norm.rmsnorm(m, W["post_feedforward_layernorm_1.weight"], eps, False)
    probs, topv, topi = route_gemma4(h, W, top_k, eps)
    if stats is not None:
        stats(probs, topv, topi)
    e = routed_experts(norm.rmsnorm(h, W["pre_feedforward_layernorm_2.weight"], eps, False), topv, topi, ex, lora_ex)
    e = norm.rmsnorm(e, W["post_feedforward_layernorm_2.weight"], eps, False)
    _, y = norm.add_rmsnorm(m, e, W["post_feedforward_layernorm.weight"], eps, False)
    return (h + y) * W["layer_scalar"]


class FrozenExpertsFn(torch.autograd.Function):
    """Frozen experts over expert-grouped rows (moe.py:110-143): apply(xs [R, H], counts, bank, group, act_name).
    bank is an Int4Experts (dequantized tile by tile inside the GEMMs) or a BF16Experts. counts may be a list (as in
    the reference) or an int32/int64 device tensor (no host sync); `group` is the reference's memory hint and is not
    needed. The backward gives dX only; it re-dequantizes the bank inside the dX GEMMs, and uses the gate/up
    pre-activations kept by the forward unless set_save_preactivations(False) (then only xs is kept, as in the
    reference, and h is recomputed)."""

    @staticmethod
    def forward(ctx, xs, counts, bank, group, act_name="silu"):
        if not isinstance(bank, (Int4Experts, BF16Experts)):
            raise _lib.SmelbError(f"FrozenExpertsFn: unsupported bank {type(bank).__name__}")
        if act_name not in _lib.ACT:
            raise ValueError(f"unknown activation {act_name}")
        xs = _bf16(xs, "FrozenExpertsFn: xs")
        dev = xs.device
        if isinstance(counts, torch.Tensor):
            counts_t = counts.to(device=dev, dtype=torch.int32).contiguous()
        else:
            if sum(counts) != xs.shape[0]:
                raise _lib.SmelbError(f"FrozenExpertsFn: counts sum to {sum(counts)}, xs has {xs.shape[0]} rows")
            counts_t = torch.tensor(list(counts), dtype=torch.int32, device=dev)
        ops = bank.kernel_operands()
        R, H = xs.shape
        int4 = "gu_q" in ops
        I = ops["dn_q"].shape[-1] * 2 if int4 else ops["fz_dn"].shape[-1]
        E = counts_t.numel()
        keep_h = ctx.needs_input_grad[0] and _SAVE_PREACT[0]
        h = torch.empty(R, 2 * I, dtype=torch.bfloat16, device=dev) if keep_h else None
        a = torch.empty(R, I, dtype=torch.bfloat16, device=dev)
        out = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
        if int4:
            _lib.call("smelb_frozen_experts_fwd", _lib.ptr(xs), R, H, I, _lib.ptr(counts_t), E, _lib.ptr(ops["gu_q"]),
                      _lib.ptr(ops["gu_sz"]), _lib.ptr(ops["dn_q"]), _lib.ptr(ops["dn_sz"]), _lib.ACT[act_name],
                      _lib.ptr(h), _lib.ptr(a), _lib.ptr(out), _lib.stream_ptr(dev))
        else:
            _lib.call("smelb_frozen_experts_bf16_fwd", _lib.ptr(xs), R, H, I, _lib.ptr(counts_t), E,
                      _lib.ptr(ops["fz_gu"]), _lib.ptr(ops["fz_dn"]), _lib.ACT[act_name], _lib.ptr(h), _lib.ptr(a),
                      _lib.ptr(out), _lib.stream_ptr(dev))
        ctx.saved = (xs, h, counts_t, ops, I, act_name)
        return out

    @staticmethod
    def backward(ctx, dy):
        xs, h, counts_t, ops, I, act_name = ctx.saved
        dy = dy.to(torch.bfloat16).contiguous()
        R, H = xs.shape
        dev = xs.device
        dh = torch.empty(R, 2 * I, dtype=torch.bfloat16, device=dev)
        dx = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
        h_buf = torch.empty(R, 2 * I, dtype=torch.bfloat16, device=dev) if h is None else None
        if "gu_q" in ops:
            _lib.call("smelb_frozen_experts_bwd", _lib.ptr(xs), _lib.ptr(dy), R, H, I, _lib.ptr(counts_t),
                      counts_t.numel(), _lib.ptr(ops["gu_q"]), _lib.ptr(ops["gu_sz"]), _lib.ptr(ops["dn_q"]),
                      _lib.ptr(ops["dn_sz"]), _lib.ACT[act_name], _lib.ptr(h), _lib.ptr(h_buf), _lib.ptr(dh),
                      _lib.ptr(dx), _lib.stream_ptr(dev))
        else:
            _lib.call("smelb_frozen_experts_bf16_bwd", _lib.ptr(xs), _lib.ptr(dy), R, H, I, _lib.ptr(counts_t),
                      counts_t.numel(), _lib.ptr(ops["fz_gu"]), _lib.ptr(ops["fz_dn"]), _lib.ACT[act_name],
                      _lib.ptr(h), _lib.ptr(h_buf), _lib.ptr(dh), _lib.ptr(dx), _lib.stream_ptr(dev))
        return dx, None, None, None, None
