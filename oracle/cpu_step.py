"""CPU baseline of the benchmark step — TEST / BASELINE INFRASTRUCTURE ONLY (used by bench.py's CPU leg and the
reference arm; never by the product).

It restates the reference's own CPU execution of the MoE layer (smel/moe.py on a CPU tensor): the router, the
stable-sort dispatch, frozen experts dequantized group by group (`expert_group` experts at a time, smel/moe.py:75-85
and smel/quant.py:87-94) in every pass, a per-expert matmul loop (smel/moe.py:67-72), selected experts with LoRA,
the shared expert with LoRA and the fp32 combine; then a recompute under autograd and the backward, in which the
frozen experts are dequantized again for dX (smel/moe.py:128-143). One step = forward (no grad) + recompute +
backward, as in the benchmark.
"""
import numpy as np
import torch
import torch.nn.functional as F

from . import moe_oracle as O


def _dequant_group(q, s, z, dtype):
    # smel/quant.py:87-94 with the compute dtype of the layer
    codes = torch.stack((q & 0xF, q >> 4), dim=-1).reshape(*q.shape[:-1], s.shape[-1], -1).to(dtype)
    w = codes * s.unsqueeze(-1).to(dtype) + z.unsqueeze(-1).to(dtype)
    return w.reshape(*q.shape[:-1], -1)


class _FrozenCPU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xs, counts, bank, group, act_name):
        ctx.save_for_backward(xs)
        ctx.counts, ctx.bank, ctx.group, ctx.act = counts, bank, group, act_name
        out = xs.new_empty(xs.shape)
        for e0, e1, r0, r1, sub in _groups(counts, group):
            gu, dn = _weights(bank, e0, e1, xs.dtype)
            h = _loop_mm(xs[r0:r1], gu, sub)
            g, u = h.chunk(2, dim=-1)
            out[r0:r1] = _loop_mm(O.act(g, act_name) * u, dn, sub)
        return out

    @staticmethod
    def backward(ctx, dy):
        (xs,) = ctx.saved_tensors
        dx = torch.zeros_like(xs)
        for e0, e1, r0, r1, sub in _groups(ctx.counts, ctx.group):
            gu, dn = _weights(ctx.bank, e0, e1, xs.dtype)
            g, u = _loop_mm(xs[r0:r1], gu, sub).float().chunk(2, dim=-1)
            da = _loop_mm(dy[r0:r1], dn, sub, transpose=False).float()
            a, dadg = O.act_and_grad(g, ctx.act)
            dh = torch.cat([da * u * dadg, da * a], dim=-1).to(xs.dtype)
            dx[r0:r1] = _loop_mm(dh, gu, sub, transpose=False)
        return dx, None, None, None, None


def _groups(counts, group):
    row = 0
    for e0 in range(0, len(counts), group):
        sub = counts[e0:e0 + group]
        n = sum(sub)
        if n:
            yield e0, min(len(counts), e0 + group), row, row + n, sub
        row += n


def _weights(bank, e0, e1, dtype):
    return (_dequant_group(bank["gu_q"][e0:e1], bank["gu_s"][e0:e1], bank["gu_z"][e0:e1], dtype),
            _dequant_group(bank["dn_q"][e0:e1], bank["dn_s"][e0:e1], bank["dn_z"][e0:e1], dtype))


def _loop_mm(x, w, counts, transpose=True):
    outs, s = [], 0
    for g, c in enumerate(counts):
        if c:
            outs.append(x[s:s + c] @ (w[g].t() if transpose else w[g]))
            s += c
    return torch.cat(outs) if outs else x.new_zeros(0, w.shape[1] if transpose else w.shape[2])


def layer_forward(x, W, bank, sel, sel_gu, sel_dn, lex, lsh, K, group=32, act_name="silu"):
    """One MoE layer forward on the CPU (differentiable in x and the LoRA tensors)."""
    logits = F.linear(x, W["mlp.gate.weight"])
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    topv, topi = torch.topk(probs, K, dim=-1)
    topv = (topv / topv.sum(-1, keepdim=True)).to(x.dtype)
    N, H = x.shape
    E = bank["gu_q"].shape[0]
    flat = topi.reshape(-1)
    order = torch.argsort(flat, stable=True)
    tok = order // K
    counts = torch.bincount(flat, minlength=E).tolist()
    xs = x[tok]
    slot = {int(e): j for j, e in enumerate(sel)}
    counts_f = [0 if e in slot else c for e, c in enumerate(counts)]
    e_sorted = flat[order]
    sel_mask = torch.zeros(E, dtype=torch.bool)
    sel_mask[list(slot)] = True
    fr_rows = (~sel_mask[e_sorted]).nonzero().squeeze(1)
    rows, vals = [fr_rows], [_FrozenCPU.apply(xs[fr_rows], counts_f, bank, group, act_name)]
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    for e, j in slot.items():
        c = counts[e]
        if c:
            r0 = int(starts[e])
            L = {k: (v[j] if k != "scale" else v) for k, v in lex.items()}
            I = sel_dn.shape[2]
            rows.append(torch.arange(r0, r0 + c))
            vals.append(O.mlp(xs[r0:r0 + c], sel_gu[j][:I], sel_gu[j][I:], sel_dn[j], L, act_name).to(x.dtype))
    y = x.new_zeros(xs.shape[0], H).index_put((torch.cat(rows),), torch.cat(vals))
    inv = torch.empty_like(order)
    inv[order] = torch.arange(order.numel())
    routed = (y[inv].view(N, K, H).float() * topv.float().unsqueeze(-1)).sum(1).to(x.dtype)
    pre = "mlp.shared_expert."
    sh = O.mlp(x, W[pre + "gate_proj.weight"], W[pre + "up_proj.weight"], W[pre + "down_proj.weight"], lsh, "silu")
    return routed + sh * torch.sigmoid(F.linear(x, W["mlp.shared_expert_gate.weight"]))


def prepare(layer, dtype=torch.float32, tokens=None):
    """CPU copies of a synthetic layer (smelb.synth.qwen_layer output) for the baseline: bf16 weights cast to `dtype`,
    the int4 bank kept packed, LoRA tensors as leaf tensors requiring grad. `tokens` takes the first rows of x."""
    ex = layer["ex"]
    bank = {"gu_q": ex.frozen.gu["q"], "gu_s": ex.frozen.gu["scale"], "gu_z": ex.frozen.gu["zero"],
            "dn_q": ex.frozen.dn["q"], "dn_s": ex.frozen.dn["scale"], "dn_z": ex.frozen.dn["zero"]}
    return prepare_parts(layer["x"], layer["W"], bank, layer["meta"]["selected"], ex.sel_gate_up, ex.sel_down,
                         layer["lora"], layer["meta"]["K"], dtype, tokens)


def prepare_tensors(t, dtype=torch.float32, tokens=None):
    """The same from smelb.synth.qwen_layer_tensors output (the bf16 bank before quantization): the bank is
    quantized with the reference's algorithm (moe_oracle.quantize_int4, as torch operations on the bank's device),
    so building the baseline's inputs runs nothing of libsmelb."""
    gu, dn, sel = t["gate_up"], t["down"], t["sel"]
    on_dev = gu.is_cuda
    qg = O.quantize_int4(gu, 64, on_device=on_dev)
    qd = O.quantize_int4(dn, 64, on_device=on_dev)
    bank = {"gu_q": qg["q"], "gu_s": qg["scale"], "gu_z": qg["zero"],
            "dn_q": qd["q"], "dn_s": qd["scale"], "dn_z": qd["zero"]}
    return prepare_parts(t["x"], t["W"], bank, sel, gu[sel], dn[sel], t["lora"], t["meta"]["K"], dtype, tokens)


def prepare_parts(x, W, bank, sel, sel_gu, sel_dn, lora, K, dtype=torch.float32, tokens=None):
    names = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")
    x = x[:tokens] if tokens else x
    lex = {n: getattr(lora.experts, n).detach().cpu().to(dtype).requires_grad_(True) for n in names}
    lex["scale"] = lora.experts.scale
    lsh = {n: getattr(lora.shared, n).detach().cpu().to(dtype).requires_grad_(True) for n in names}
    lsh["scale"] = lora.shared.scale
    return {"x": x.detach().cpu().to(dtype), "W": {k: v.detach().cpu().to(dtype) for k, v in W.items()},
            "bank": {k: v.cpu() for k, v in bank.items()}, "sel": list(sel), "sel_gu": sel_gu.cpu().to(dtype),
            "sel_dn": sel_dn.cpu().to(dtype), "lex": lex, "lsh": lsh, "K": K}


def step(p, gy):
    """Forward (no grad), recompute under autograd, backward. Returns dX."""
    with torch.no_grad():
        layer_forward(p["x"], p["W"], p["bank"], p["sel"], p["sel_gu"], p["sel_dn"], p["lex"], p["lsh"], p["K"])
    x = p["x"].clone().requires_grad_(True)
    out = layer_forward(x, p["W"], p["bank"], p["sel"], p["sel_gu"], p["sel_dn"], p["lex"], p["lsh"], p["K"])
    out.backward(gy)
    return x.grad
