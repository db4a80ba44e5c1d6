"""Seeded synthetic MoE layers of the benchmark configurations (no checkpoints or datasets are needed).

gemma_layer(): the Gemma-4-26B-A4B-like MoE block (H 2816, 128 experts, top-8, expert intermediate 704, dense GeGLU
MLP 2112 with LoRA, the four feed-forward norms and the Gemma router) with the same kind of Zipf skew, applied through
the router's RMSNorm prologue (h += mu * u, a rank-1 router component along u).

qwen_layer(): the Qwen3.6-35B-A3B layer shape (H 2048, 256 experts, top-8, expert intermediate 512, shared expert 512
with a sigmoid gate). Router logits are skewed Zipf-like over a seeded expert permutation: a rank-1 component
b_e = -s * tau * ln(rank_e) is added to the router (W_g += b/mu * u, x += mu * u for a seeded unit vector u), with tau
bisected so that the 12 top-ranked experts hold `share` (default 50%) of the renormalised top-k gate mass. Those 12
experts are the selected bf16 experts with LoRA; all experts are also packed int4 group-64 (the frozen bank).
Weights ~ N(0, 0.02), hidden states ~ N(0, 1), LoRA A with the PEFT init and B ~ N(0, 0.02).
"""
import torch

from .lora import ExpertsLoRA, LayerLoRA, MLPLoRA
from .moe import Int4Experts, LayerExperts


def packed_lengths(total, lo=64, hi=1024, seed=0):
    """Sequence lengths drawn uniformly in [lo, hi] until the next would exceed `total`; the remainder is appended
    (merged into the previous sequence when shorter than lo). Returns (lengths, cu_seqlens)."""
    g = torch.Generator().manual_seed(seed)
    lens, used = [], 0
    while True:
        n = int(torch.randint(lo, hi + 1, (1,), generator=g))
        if used + n > total:
            break
        lens.append(n)
        used += n
    rest = total - used
    if rest:
        if rest < lo and lens:
            lens[-1] += rest
        else:
            lens.append(rest)
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    return lens, torch.tensor(cu, dtype=torch.int32)


def _share_of_top(logits, ranked, n_top, k):
    probs = torch.softmax(logits.float(), -1)
    topv, topi = probs.topk(k, -1)
    topv = topv / topv.sum(-1, keepdim=True)
    top_set = torch.zeros(logits.shape[1], dtype=torch.bool, device=logits.device)
    top_set[ranked[:n_top]] = True
    return float((topv * top_set[topi]).sum() / topv.sum())


def qwen_layer_tensors(T=4092, H=2048, E=256, K=8, I=512, S=512, n_sel=12, r=16, alpha=32.0, zipf_s=1.1,
                       share=0.5, seed=0, device="cuda", mu=4.0, uniform=False, with_lora=True, tau=None):
    """The seeded tensors of one synthetic layer, built with torch operations only (nothing of libsmelb runs, so a
    process that only needs the inputs, such as the benchmark's CPU reference arm, never loads the library):
    x [T, H] bf16, W (router / shared tensors, bf16), the bf16 bank gate_up [E, 2I, H] / down [E, H, I] before
    quantization, the selected expert ids, LoRA modules (or None) and meta."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)

    def rnd(*s, std=0.02):
        return torch.randn(*s, generator=g, device=dev) * std

    x = rnd(T, H, std=1.0)
    wg = rnd(E, H)
    W = {"mlp.shared_expert.gate_proj.weight": rnd(S, H).bfloat16(),
         "mlp.shared_expert.up_proj.weight": rnd(S, H).bfloat16(),
         "mlp.shared_expert.down_proj.weight": rnd(H, S).bfloat16(),
         "mlp.shared_expert_gate.weight": rnd(1, H).bfloat16()}
    W["mlp.shared_expert.gate_up_proj.weight"] = torch.cat((W["mlp.shared_expert.gate_proj.weight"],
                                                            W["mlp.shared_expert.up_proj.weight"]))
    gu = rnd(E, 2 * I, H).bfloat16()
    dn = rnd(E, H, I).bfloat16()
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed + 1))  # perm[0] = rank-1 expert
    tau = None if tau is None else float(tau)  # fixed Zipf temperature, or bisected below
    meta = {"seed": seed, "T": T, "H": H, "E": E, "K": K, "I": I, "S": S, "n_sel": n_sel, "r": r, "alpha": alpha}
    if not uniform:
        u = torch.randn(H, generator=g, device=dev)
        u = u / u.norm()
        rank = torch.empty(E, device=dev)
        rank[perm.to(dev)] = torch.arange(1, E + 1, device=dev, dtype=torch.float32)
        xs = x + mu * u
        lo_t, hi_t = 0.0, 4.0
        for _ in range(24 if tau is None else 0):  # bisection on tau for the target top-12 share
            tau = 0.5 * (lo_t + hi_t)
            b = -zipf_s * tau * torch.log(rank)
            logits = (xs.bfloat16() @ (wg + (b / mu)[:, None] * u[None]).bfloat16().t())
            sh = _share_of_top(logits, perm.to(dev), n_sel, K)
            if sh < share:
                lo_t = tau
            else:
                hi_t = tau
        if tau is None:
            tau = 0.5 * (lo_t + hi_t)
        b = -zipf_s * tau * torch.log(rank)
        wg = wg + (b / mu)[:, None] * u[None]
        x = xs
        meta.update(tau=float(tau), share=_share_of_top(x.bfloat16() @ wg.bfloat16().t(), perm.to(dev), max(n_sel, 1), K),
                    zipf_s=zipf_s, mu=mu)
    W["mlp.gate.weight"] = wg.bfloat16()
    sel = perm[:n_sel].tolist() if n_sel else []
    lora = None
    if with_lora:
        torch.manual_seed(seed)  # PEFT init of A draws from the global generator
        le = ExpertsLoRA(sel, H, I, r, alpha).to(dev) if sel else None
        ls = MLPLoRA(H, S, r, alpha).to(dev)
        gb = torch.Generator(device=dev).manual_seed(seed + 2)
        with torch.no_grad():
            for mod in (le, ls):
                if mod is None:
                    continue
                for n, p in mod.named_parameters():
                    if n.startswith("B_"):
                        p.copy_(torch.randn(p.shape, generator=gb, device=dev) * 0.02)
        lora = LayerLoRA(le, ls)
    lens, cu = packed_lengths(T, seed=seed)
    meta["n_seqs"] = len(lens)
    meta["selected"] = sel
    return {"x": x.bfloat16().contiguous(), "W": W, "gate_up": gu, "down": dn, "sel": sel, "lora": lora,
            "meta": meta, "cu_seqlens": cu}


def qwen_layer(T=4092, H=2048, E=256, K=8, I=512, S=512, n_sel=12, r=16, alpha=32.0, zipf_s=1.1, share=0.5,
               seed=0, device="cuda", mu=4.0, uniform=False, with_lora=True, keep_bf16=False, tau=None):
    """Build one synthetic layer: qwen_layer_tensors with the bank quantized int4 group-64 by the CUDA quantizer.
    Returns a dict with x [T, H] bf16, W (router / shared tensors, bf16), ex (LayerExperts), lora (LayerLoRA or
    None), meta, and with keep_bf16 the bank before quantization (bank_bf16)."""
    t = qwen_layer_tensors(T=T, H=H, E=E, K=K, I=I, S=S, n_sel=n_sel, r=r, alpha=alpha, zipf_s=zipf_s, share=share,
                           seed=seed, device=device, mu=mu, uniform=uniform, with_lora=with_lora, tau=tau)
    gu, dn, sel = t["gate_up"], t["down"], t["sel"]
    bank = Int4Experts.from_bf16(gu, dn, 64)
    ex = LayerExperts(bank, sel if sel else None, gu[sel].clone() if sel else None, dn[sel].clone() if sel else None)
    out = {"x": t["x"], "W": t["W"], "ex": ex, "lora": t["lora"], "meta": t["meta"], "cu_seqlens": t["cu_seqlens"]}
    if keep_bf16:
        out["bank_bf16"] = (gu, dn)
    return out


def gemma_layer_tensors(T=4096, H=2816, E=128, K=8, I=704, S=2112, n_sel=12, r=16, alpha=32.0, zipf_s=1.1,
                        share=0.5, seed=0, device="cuda", mu=4.0, eps=1e-6, with_lora=True):
    """Seeded tensors of one synthetic Gemma 4 MoE block (torch operations only): h, xm [T, H] bf16; W with the dense
    MLP (gate / up / down and the stacked gate_up), router.scale ~ N(1, 0.2), router.proj.weight, per_expert_scale
    ~ U(0.5, 1.5), the four feed-forward norm weights ~ N(1, 0.2), layer_scalar ~ U(0.7, 1.3); the bf16 bank; the
    selected ids (the 12 top-ranked experts); LoRA modules (experts, and the dense MLP as "shared"); meta."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)

    def rnd(*s, std=0.02, mean=0.0):
        return torch.randn(*s, generator=g, device=dev) * std + mean

    h = rnd(T, H, std=1.0)
    xm = rnd(T, H, std=1.0)
    W = {"mlp.gate_proj.weight": rnd(S, H).bfloat16(), "mlp.up_proj.weight": rnd(S, H).bfloat16(),
         "mlp.down_proj.weight": rnd(H, S).bfloat16(), "router.scale": rnd(H, std=0.2, mean=1.0).bfloat16()}
    W["mlp.gate_up_proj.weight"] = torch.cat((W["mlp.gate_proj.weight"], W["mlp.up_proj.weight"]))
    for n in ("pre_feedforward_layernorm_2", "post_feedforward_layernorm_1", "post_feedforward_layernorm_2",
              "post_feedforward_layernorm"):
        W[n + ".weight"] = rnd(H, std=0.2, mean=1.0).bfloat16()
    W["router.per_expert_scale"] = (torch.rand(E, generator=g, device=dev) + 0.5).bfloat16()
    W["layer_scalar"] = (torch.rand(1, generator=g, device=dev) * 0.6 + 0.7).bfloat16()
    proj = rnd(E, H)
    gu = rnd(E, 2 * I, H).bfloat16()
    dn = rnd(E, H, I).bfloat16()
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed + 1))
    u = torch.randn(H, generator=g, device=dev)
    u = u / u.norm()
    rank = torch.empty(E, device=dev)
    rank[perm.to(dev)] = torch.arange(1, E + 1, device=dev, dtype=torch.float32)
    hs = h + mu * u
    scale = W["router.scale"].float()

    def logits_of(pw):  # the router of smel/moe.py:170-177 (bf16 steps), for the calibration only
        x = (hs * torch.rsqrt(hs.pow(2).mean(-1, keepdim=True) + eps)).bfloat16()
        x = (x * W["router.scale"] * H ** -0.5).bfloat16()
        return x @ pw.bfloat16().t()

    f = float((scale * u * u).sum()) / H ** 0.5  # logit shift per unit rank-1 weight along u
    lo_t, hi_t, tau = 0.0, 4.0, None
    for _ in range(24):
        tau = 0.5 * (lo_t + hi_t)
        b = -zipf_s * tau * torch.log(rank)
        sh = _share_of_top(logits_of(proj + (b / (mu * f))[:, None] * u[None]), perm.to(dev), n_sel, K)
        if sh < share:
            lo_t = tau
        else:
            hi_t = tau
    tau = 0.5 * (lo_t + hi_t)
    proj = proj + (-zipf_s * tau * torch.log(rank) / (mu * f))[:, None] * u[None]
    W["router.proj.weight"] = proj.bfloat16()
    meta = {"seed": seed, "T": T, "H": H, "E": E, "K": K, "I": I, "S": S, "n_sel": n_sel, "r": r, "alpha": alpha,
            "eps": eps, "tau": float(tau), "zipf_s": zipf_s, "mu": mu,
            "share": _share_of_top(logits_of(proj), perm.to(dev), max(n_sel, 1), K)}
    sel = perm[:n_sel].tolist() if n_sel else []
    lora = None
    if with_lora:
        torch.manual_seed(seed)
        le = ExpertsLoRA(sel, H, I, r, alpha).to(dev) if sel else None
        ls = MLPLoRA(H, S, r, alpha).to(dev)
        gb = torch.Generator(device=dev).manual_seed(seed + 2)
        with torch.no_grad():
            for mod in (le, ls):
                if mod is None:
                    continue
                for n, p in mod.named_parameters():
                    if n.startswith("B_"):
                        p.copy_(torch.randn(p.shape, generator=gb, device=dev) * 0.02)
        lora = LayerLoRA(le, ls)
    meta["selected"] = sel
    return {"h": hs.bfloat16().contiguous(), "xm": xm.bfloat16().contiguous(), "W": W, "gate_up": gu, "down": dn,
            "sel": sel, "lora": lora, "meta": meta}


def gemma_layer(T=4096, H=2816, E=128, K=8, I=704, S=2112, n_sel=12, r=16, alpha=32.0, zipf_s=1.1, share=0.5,
                seed=0, device="cuda", with_lora=True, keep_bf16=False):
    """gemma_layer_tensors with the bank quantized int4 group-64 (CUDA quantizer) and the experts as LayerExperts
    (GELU-tanh)."""
    t = gemma_layer_tensors(T=T, H=H, E=E, K=K, I=I, S=S, n_sel=n_sel, r=r, alpha=alpha, zipf_s=zipf_s, share=share,
                            seed=seed, device=device, with_lora=with_lora)
    gu, dn, sel = t["gate_up"], t["down"], t["sel"]
    bank = Int4Experts.from_bf16(gu, dn, 64)
    ex = LayerExperts(bank, sel if sel else None, gu[sel].clone() if sel else None, dn[sel].clone() if sel else None,
                      act="gelu_tanh")
    out = {"h": t["h"], "xm": t["xm"], "W": t["W"], "ex": ex, "lora": t["lora"], "meta": t["meta"]}
    if keep_bf16:
        out["bank_bf16"] = (gu, dn)
    return out


def flops_per_token(H, E, K, I, S, n_lora_rows_frac=0.0, r=16):
    """Algorithmic forward FLOPs per token of the layer: routed gate_up + down (2*K*3*H*I), shared (2*3*H*S),
    router (2*H*E), plus the LoRA products on the fraction of routed rows that hit LoRA experts and on the shared
    expert (2*r*(3H + 3I) per LoRA row)."""
    base = 2 * K * 3 * H * I + 2 * 3 * H * S + 2 * H * E
    lora = 2 * r * (2 * H + 2 * I + I + H)  # xA (gate, up), (xA)B (gate, up), aA, (aA)B
    return base + (K * n_lora_rows_frac) * lora + lora * (S / max(I, 1))


def int4_bank_bytes_per_expert(H, I):
    """Bytes the fused GEMMs read per frozen expert per pass: nibbles (3 H I / 2) + (scale, zero) (3 H I / 64 * 4)."""
    return 3 * H * I // 2 + 3 * H * I // 64 * 4


def lengths_summary(cu):
    return {"n_seqs": int(cu.numel() - 1), "max_len": int((cu[1:] - cu[:-1]).max())}


__all__ = ["gemma_layer", "gemma_layer_tensors", "qwen_layer", "qwen_layer_tensors", "packed_lengths", "flops_per_token", "int4_bank_bytes_per_expert"]
