"""CPU oracle for the smelb MoE layer — TEST INFRASTRUCTURE ONLY.

A restatement, on the CPU, of the reference algorithm of SMEL FT's MoE expert layer (smel/moe.py, smel/quant.py,
smel/lora.py of the smel-ft source tree). Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use it,
as the checker / baseline; the product (smel-ft_b200/smelb) never imports it.

Integer and byte work (int4 pack / unpack, the stable dispatch permutation) is numpy; floating-point work is torch on
the CPU in the dtype the caller passes (fp32 for parity, fp64 for tight checks), with gradients by torch autograd of
the same forward math. Each function names the reference lines it restates.

Pinning: tests/golden/*.pt hold input/output vectors produced by the reference itself (tests/golden/make_golden.py,
run where the reference is importable); tests/test_oracle.py checks this oracle against them.
"""
import math

import numpy as np
import torch
import torch.nn.functional as F

GELU_C = 0.7978845608028654  # sqrt(2 / pi)


# ============================================================================================== int4 format
def quantize_int4(w: torch.Tensor, group: int = 64, clip_search=(1.0, 0.95, 0.9, 0.85, 0.8),
                  on_device: bool = False) -> dict:
    """smel/quant.py:5-44. Per group of `group` values along the last dim: try each clip factor c (range shrunk
    towards the group midpoint), scale = bf16(max((hi - lo) / 15, 1e-8)), zero = bf16(lo),
    q = clamp(round((w - zero) / scale), 0, 15); keep the first c with the smallest squared error.
    Packs two codes per byte, the even column in the low nibble. on_device: run the same torch operations on w's
    device (used to build large synthetic banks quickly) and return CPU tensors."""
    w = w.detach() if on_device else w.detach().cpu()
    if w.dim() == 3 and w.shape[0] > 16:
        parts = [quantize_int4(w[i:i + 16], group, clip_search, on_device) for i in range(0, w.shape[0], 16)]
        return {k: torch.cat([p[k] for p in parts]) for k in parts[0]}
    K = w.shape[-1]
    assert K % group == 0 and group % 2 == 0
    wg = w.float().reshape(*w.shape[:-1], K // group, group)
    lo0 = wg.amin(-1, keepdim=True)
    hi0 = wg.amax(-1, keepdim=True)
    mid = (lo0 + hi0) / 2
    best = None
    for c in clip_search:
        lo = mid + (lo0 - mid) * c
        hi = mid + (hi0 - mid) * c
        scale = ((hi - lo) / 15).clamp_min(1e-8).to(torch.bfloat16).float()
        zero = lo.to(torch.bfloat16).float()
        q = torch.round((wg - zero) / scale).clamp_(0, 15)
        err = (q * scale + zero - wg).pow(2).sum(-1, keepdim=True)
        if best is None:
            best = [err, q, scale, zero]
        else:
            m = err < best[0]
            best = [torch.where(m, err, best[0]), torch.where(m, q, best[1]), torch.where(m, scale, best[2]),
                    torch.where(m, zero, best[3])]
    codes = best[1].to(torch.uint8).reshape(*w.shape[:-1], K)
    if on_device:  # the same packing as pack_nibbles, as torch operations
        packed = (codes[..., 0::2] | (codes[..., 1::2] << 4)).cpu()
    else:
        packed = torch.from_numpy(pack_nibbles(codes.numpy()))
    return {"q": packed, "scale": best[2].squeeze(-1).to(torch.bfloat16).cpu(),
            "zero": best[3].squeeze(-1).to(torch.bfloat16).cpu()}


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """codes uint8 [..., K] (0..15) -> bytes [..., K/2]; byte j = codes[2j] | codes[2j+1] << 4 (quant.py:42)."""
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(q: np.ndarray) -> np.ndarray:
    """bytes [..., K/2] -> codes [..., K]: column 2j = low nibble, 2j+1 = high nibble (quant.py:58-65, 90-92)."""
    q = np.asarray(q, dtype=np.uint8)
    out = np.empty(q.shape[:-1] + (q.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = q & 0xF
    out[..., 1::2] = q >> 4
    return out


def dequant_int4(q, scale, zero, dtype=torch.float32) -> torch.Tensor:
    """codes * scale + zero computed in fp32 (quant.py:63-64 / :87-94 with fp32 compute), then cast once."""
    codes = torch.from_numpy(unpack_nibbles(q.cpu().numpy() if isinstance(q, torch.Tensor) else q)).float()
    s, z = scale.cpu().float(), zero.cpu().float()
    G = s.shape[-1]
    K = codes.shape[-1]
    w = codes.reshape(*codes.shape[:-1], G, K // G) * s.unsqueeze(-1) + z.unsqueeze(-1)
    return w.reshape(*codes.shape[:-1], K).to(dtype)


def dequant_int4_stepwise(q, scale, zero, dtype=torch.bfloat16) -> torch.Tensor:
    """smel/quant.py:87-94 dequant_int4_torch as torch runs it in `dtype`: codes cast to dtype, times scale (rounded
    to dtype), plus zero (rounded again). In bf16 this differs from dequant_int4 on many weights."""
    codes = torch.from_numpy(unpack_nibbles(q.cpu().numpy() if isinstance(q, torch.Tensor) else q))
    G = scale.shape[-1]
    K = codes.shape[-1]
    w = codes.reshape(*codes.shape[:-1], G, K // G).to(dtype)
    w = w * scale.cpu().unsqueeze(-1).to(dtype) + zero.cpu().unsqueeze(-1).to(dtype)
    return w.reshape(*codes.shape[:-1], K)


# ============================================================================================== routing
def route(x, gate_w, top_k, logits_dtype=None):
    """smel/moe.py:162-167: logits = x W^T (in the activation dtype), probs = softmax_fp32, top-k, renormalised in
    fp32, cast back to the logits dtype. Ties in probs go to the smaller expert id (a stable descending sort)."""
    logits = F.linear(x, gate_w)
    if logits_dtype is not None:
        logits = logits.to(logits_dtype)
    return route_from_logits(logits, top_k)


def route_from_logits(logits, top_k):
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    topi = topk_stable(probs, top_k)
    topv = probs.gather(1, topi)
    topv = topv / topv.sum(dim=-1, keepdim=True)
    return probs, topv.to(logits.dtype), topi


def topk_stable(probs, k):
    """Top-k indices ordered by value descending, ties by ascending index (numpy stable sort on -probs)."""
    p = probs.detach().cpu().double().numpy()
    idx = np.argsort(-p, axis=-1, kind="stable")[..., :k]
    return torch.from_numpy(idx.astype(np.int64))


def forced_route(logits_or_probs, topi, from_probs=False):
    """Routing weights at given expert choices (tests/helpers.py:89-106 patch_hf_routing): probs gathered at topi and
    renormalised."""
    probs = logits_or_probs if from_probs else torch.softmax(logits_or_probs, dim=-1, dtype=torch.float32)
    top = probs.gather(1, topi)
    return probs, top / top.sum(dim=-1, keepdim=True)


# ============================================================================================== dispatch
def dispatch(topi: np.ndarray, E: int):
    """smel/moe.py:218-223: order = stable argsort of topi.reshape(-1); tok = order // K; counts = bincount."""
    topi = np.asarray(topi)
    K = topi.shape[1]
    flat = topi.reshape(-1)
    order = np.argsort(flat, kind="stable").astype(np.int64)
    counts = np.bincount(flat, minlength=E).astype(np.int64)
    return order, order // K, counts


def dispatch_padded(topi: np.ndarray, E: int, sel_mask: np.ndarray, pad: int = 64):
    """The dispatch layout of the fused path: experts in id order, selected experts' segments padded to `pad` rows.
    Returns (counts, gcounts, offsets, row_of [T*K], src_of [total] with -1 on padding rows)."""
    flat = np.asarray(topi).reshape(-1)
    counts = np.bincount(flat, minlength=E).astype(np.int64)
    gcounts = np.where(sel_mask.astype(bool), (counts + pad - 1) // pad * pad, counts)
    offsets = np.concatenate([[0], np.cumsum(gcounts)[:-1]]).astype(np.int64)
    row_of = np.empty(flat.shape[0], dtype=np.int64)
    src_of = -np.ones(int(gcounts.sum()), dtype=np.int64)
    seen = np.zeros(E, dtype=np.int64)
    for i, e in enumerate(flat):  # stable: choices of one expert keep (t, k) order
        r = offsets[e] + seen[e]
        seen[e] += 1
        row_of[i] = r
        src_of[r] = i
    return counts, gcounts, offsets, row_of, src_of


# ============================================================================================== experts
def act(x, name):
    """smel/moe.py:91-96"""
    if name == "silu":
        return F.silu(x)
    if name == "gelu_tanh":
        return F.gelu(x, approximate="tanh")
    raise ValueError(f"unknown activation {name}")


def act_and_grad(g, name):
    """smel/moe.py:99-107: (act(g), d act / d g) in the dtype of g."""
    if name == "silu":
        sg = torch.sigmoid(g)
        return g * sg, sg * (1 + g * (1 - sg))
    t = torch.tanh(GELU_C * (g + 0.044715 * g ** 3))
    return 0.5 * g * (1 + t), 0.5 * (1 + t) + 0.5 * g * (1 - t * t) * GELU_C * (1 + 3 * 0.044715 * g * g)


def frozen_experts(xs, counts, gu, dn, act_name="silu"):
    """smel/moe.py:110-117 (per-expert loop of _gmm, moe.py:67-72): rows grouped by expert; gu [E, 2I, H],
    dn [E, H, I] (already dequantized)."""
    outs, s = [], 0
    for e, c in enumerate(list(counts)):
        c = int(c)
        if c:
            h = xs[s:s + c] @ gu[e].t()
            g, u = h.chunk(2, dim=-1)
            outs.append((act(g, act_name) * u) @ dn[e].t())
            s += c
    return torch.cat(outs) if outs else xs.new_zeros(0, dn.shape[1])


def frozen_experts_backward(xs, dy, counts, gu, dn, act_name="silu"):
    """smel/moe.py:128-143: dx of the frozen experts (no weight gradients)."""
    dxs, s = [], 0
    for e, c in enumerate(list(counts)):
        c = int(c)
        if c:
            h = xs[s:s + c] @ gu[e].t()
            g, u = h.chunk(2, dim=-1)
            da = dy[s:s + c] @ dn[e]
            a, dadg = act_and_grad(g, act_name)
            dh = torch.cat([da * u * dadg, da * a], dim=-1)
            dxs.append(dh @ gu[e])
            s += c
    return torch.cat(dxs) if dxs else xs.new_zeros(0, xs.shape[1])


def lora_linear(x, w, A, B, scale):
    """smel/lora.py:61-69: x W^T + scale (x A^T) B^T."""
    y = x @ w.t()
    if A is None:
        return y
    return y + scale * ((x @ A.to(x.dtype).t()) @ B.to(x.dtype).t())


def lora_gate_up(x, w_gate_up, A_gate, B_gate, A_up, B_up, scale):
    """smel/lora.py:72-83: (gate, up) over the stacked weight, each half with its LoRA pair."""
    I = w_gate_up.shape[0] // 2
    return (lora_linear(x, w_gate_up[:I], A_gate, B_gate, scale), lora_linear(x, w_gate_up[I:], A_up, B_up, scale))


def mlp(x, w_gate, w_up, w_down, lora, act_name="silu"):
    """smel/moe.py:183-194 (gate and up through lora_linear, smel/lora.py:72-83 is the same math stacked).
    lora: None or dict with A_gate, B_gate, A_up, B_up, A_down, B_down, scale."""
    L = lora or {}
    s = L.get("scale", 0.0)
    g = lora_linear(x, w_gate, L.get("A_gate"), L.get("B_gate"), s)
    u = lora_linear(x, w_up, L.get("A_up"), L.get("B_up"), s)
    return lora_linear(act(g, act_name) * u, w_down, L.get("A_down"), L.get("B_down"), s)


def moe_layer(x, W, bank_gu, bank_dn, top_k, sel_ids=(), sel_gu=None, sel_dn=None, lora_ex=None, lora_sh=None,
              act_name="silu", topi=None, logits=None):
    """smel/moe.py:255-263 moe_forward (route -> routed_experts -> + shared_mlp), in the dtype of x.

    bank_gu [E, 2I, H] / bank_dn [E, H, I]: the frozen bank, dequantized. Selected experts (sel_ids, slot order) use
    sel_gu / sel_dn and per-slot LoRA (lora_ex: dict of [k, ...] tensors + scale). topi forces the expert choices
    (tests/helpers.py:89-106); logits, when given, replace x W_gate^T (to route on another implementation's logits).
    Returns (out, probs, topv, topi). Differentiable in x and the LoRA tensors (torch autograd)."""
    if logits is None:
        logits = F.linear(x, W["mlp.gate.weight"].to(x.dtype))
    probs = torch.softmax(logits.to(x.dtype), dim=-1, dtype=torch.float32)
    if topi is None:
        topi = topk_stable(probs, top_k)
    top = probs.gather(1, topi)
    topv = (top / top.sum(dim=-1, keepdim=True)).to(x.dtype)
    routed_out = routed(x, topv, topi, bank_gu, bank_dn, sel_ids, sel_gu, sel_dn, lora_ex, act_name)
    pre = "mlp.shared_expert."
    sh = mlp(x, W[pre + "gate_proj.weight"].to(x.dtype), W[pre + "up_proj.weight"].to(x.dtype),
             W[pre + "down_proj.weight"].to(x.dtype), lora_sh, "silu")
    sh = sh * torch.sigmoid(F.linear(x, W["mlp.shared_expert_gate.weight"].to(x.dtype)))  # moe.py:197-201
    return routed_out + sh, probs, topv, topi


def routed(x, topv, topi, bank_gu, bank_dn, sel_ids=(), sel_gu=None, sel_dn=None, lora_ex=None, act_name="silu"):
    """smel/moe.py:214-252 routed_experts: stable dispatch by expert, frozen experts from the dequantized bank,
    selected experts with LoRA, then the fp32 weighted sum over k in k order, in the dtype of x."""
    N, H = x.shape
    K = topi.shape[1]
    E = bank_gu.shape[0]
    order, tok, counts = dispatch(topi.numpy(), E)
    xs = x[torch.from_numpy(tok)]
    e_sorted = topi.reshape(-1)[torch.from_numpy(order)]
    slot = {int(e): j for j, e in enumerate(sel_ids)}
    y = x.new_zeros(xs.shape[0], H)
    rows_out, vals = [], []
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    for e in range(E):
        c = int(counts[e])
        if c == 0:
            continue
        r0 = int(starts[e])
        xe = xs[r0:r0 + c]
        if e in slot:  # moe.py:204-211 _selected_expert with lora.py:61-83
            j = slot[e]
            L = None if lora_ex is None else {k: (v[j] if k != "scale" else v) for k, v in lora_ex.items()}
            I = sel_dn.shape[2]
            ye = mlp(xe, sel_gu[j][:I], sel_gu[j][I:], sel_dn[j], L, act_name)
        else:
            I = bank_dn.shape[2]
            g, u = (xe @ bank_gu[e].t()).chunk(2, dim=-1)
            ye = (act(g, act_name) * u) @ bank_dn[e].t()
        rows_out.append(torch.arange(r0, r0 + c))
        vals.append(ye)
    if rows_out:
        y = y.index_put((torch.cat(rows_out),), torch.cat(vals))
    inv = torch.empty(order.shape[0], dtype=torch.long)
    inv[torch.from_numpy(order)] = torch.arange(order.shape[0])
    yk = y[inv].view(N, K, H)
    routed = (yk.float() * topv.float().unsqueeze(-1)).sum(1).to(x.dtype)  # moe.py:248-252
    return routed


# ============================================================================================== Gemma 4 block
def rmsnorm(x, w, eps, plus_one=True):
    """smel/layer_runner.py:110-121 (torch form of smel/norm.py rmsnorm): fp32 math, one rounding to x's dtype."""
    xf = x.double() if x.dtype == torch.float64 else x.float()
    if plus_one:
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        return (xf * (1.0 + w.to(xf.dtype))).type_as(x)
    xf = xf * torch.pow(xf.pow(2).mean(-1, keepdim=True) + eps, -0.5)
    return (xf if w is None else xf * w.to(xf.dtype)).type_as(x)


def add_rmsnorm(h, x, w, eps, plus_one=True):
    """smel/layer_runner.py:124-130: (h + x, rmsnorm(h + x))."""
    s = h + x
    return s, rmsnorm(s, w, eps, plus_one)


def route_gemma4(h, W, top_k, eps, topi=None):
    """smel/moe.py:170-180: weightless RMSNorm of h (rounded to h's dtype), x router.scale x H^-0.5, router.proj
    logits, fp32 softmax, top-k (value desc, id asc; or forced), renormalised, x per_expert_scale[topi]; topv fp32."""
    hf = h.float() if h.dtype != torch.float64 else h
    x = (hf * torch.pow(hf.pow(2).mean(-1, keepdim=True) + eps, -0.5)).type_as(h)
    x = x * W["router.scale"].to(h.dtype) * h.shape[-1] ** -0.5
    logits = F.linear(x, W["router.proj.weight"].to(h.dtype))
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32 if h.dtype != torch.float64 else torch.float64)
    if topi is None:
        topi = topk_stable(probs, top_k)
    topv = probs.gather(1, topi)
    topv = topv / topv.sum(dim=-1, keepdim=True)
    return probs, topv * W["router.per_expert_scale"].to(topv.dtype)[topi], topi


def moe_block_gemma4(h, xm, W, bank_gu, bank_dn, top_k, eps, sel_ids=(), sel_gu=None, sel_dn=None, lora_ex=None,
                     lora_sh=None, act_name="gelu_tanh", topi=None):
    """smel/layer_runner.py:252-261 (the Gemma 4 MoE block after the attention residual): dense MLP with the "shared"
    LoRA on xm and its post norm, route_gemma4 on h, routed experts on the pre-FFN-2 norm of h and their post norm,
    h + rmsnorm(m + e), times layer_scalar. Returns (out, probs, topv, topi)."""
    dt = h.dtype
    m = mlp(xm, W["mlp.gate_proj.weight"].to(dt), W["mlp.up_proj.weight"].to(dt), W["mlp.down_proj.weight"].to(dt),
            lora_sh, act_name)
    m = rmsnorm(m, W["post_feedforward_layernorm_1.weight"], eps, False)
    probs, topv, topi = route_gemma4(h, W, top_k, eps, topi)
    xe = rmsnorm(h, W["pre_feedforward_layernorm_2.weight"], eps, False)
    e = routed(xe, topv, topi, bank_gu, bank_dn, sel_ids, sel_gu, sel_dn, lora_ex, act_name)
    e = rmsnorm(e, W["post_feedforward_layernorm_2.weight"], eps, False)
    out = (h + rmsnorm(m + e, W["post_feedforward_layernorm.weight"], eps, False)) * W["layer_scalar"].to(dt)
    return out, probs, topv, topi


# ============================================================================================== metrics
def routing_disagreements(topi_got, logits_ref, top_k):
    """Rows whose expert set differs from the reference top-k of `logits_ref` (high precision logits of the same
    inputs), with the logit gap of each swap: the largest |logit(e_ref) - logit(e_got)| over the experts that one
    side chose and the other did not (a near-tie report: a bf16 logit moves by up to half an ulp, so only near-ties
    may flip). Returns a list of (row, gap)."""
    ref = topk_stable(torch.softmax(logits_ref.double(), -1), top_k)
    got = topi_got.cpu()
    out = []
    for t in range(got.shape[0]):
        a, b = set(got[t].tolist()), set(ref[t].tolist())
        if a != b:
            only_got = sorted(a - b)
            only_ref = sorted(b - a)
            gap = max(abs(float(logits_ref[t, i]) - float(logits_ref[t, j])) for i in only_got for j in only_ref)
            out.append((t, gap))
    return out



def rel_err(a, b) -> float:
    """||a - b|| / ||b|| (smel/quant.py:108-110)."""
    a, b = a.detach().double(), b.detach().double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def cosine(a, b) -> float:
    a, b = a.detach().double().flatten(), b.detach().double().flatten()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-300))


def kaiming_a(shape, gen):
    """PEFT's LoRA-A init (kaiming_uniform_(a=sqrt(5)) on each [r, in] matrix, smel/lora.py:8-11): uniform in
    +-1/sqrt(in)."""
    bound = 1.0 / math.sqrt(shape[-1])
    return (torch.rand(*shape, generator=gen) * 2 - 1) * bound
