"""Generate the golden fixtures of tests/golden/ by running the REFERENCE implementation (smel-ft's smel package) on
the CPU. Run where the reference source tree is available:

    python tests/golden/make_golden.py --reference /path/to/smel-ft

Outputs (torch.save dicts of CPU tensors):
  quant.pt     quantize_int4 / dequant_int4_torch(fp32) of seeded weights, an on-grid round trip
  dispatch.pt  stable argsort / bincount of expert choices with many ties
  moe_c1.pt    config 1 (tiny Qwen-class MoE block, fp32): inputs, int4 bank, routing, dispatch, forward output,
               dX and all LoRA gradients of moe_forward with an upstream gradient
  moe_c1_bf16.pt  the same block run by the reference in bf16 on the CPU
  frozen_gelu.pt  FrozenExpertsFn forward/backward with GELU-tanh, uneven counts and an empty expert
                  (the case of the reference test tests/test_gemma4.py:153-169)
  gemma_block.pt  the Gemma 4 MoE block of smel/layer_runner.py:252-261 (dense GeGLU MLP with LoRA, route_gemma4,
                  int4 + LoRA routed experts, the four Gemma norms, layer_scalar) in fp32: inputs, outputs, routing,
                  dh, dxm and all LoRA gradients
  pack.pt      smel/pack.py: pack_layer of a small checkpoint layer (dense fp32 tensors, an A_log, an integer
               tensor, the fused bank, two selected experts) and merge_experts / merge_mlp with LoRA deltas
               (python tests/golden/make_golden.py --only pack writes just this file)
  ce.pt        smel/loss.py chunked_ce in bf16 on the CPU (loss and dL/dh) for a bf16 head with ragged vocabulary
               and token chunks, the same head as int8 rows (with quantize_int8_rows' q / scale), and a softcapped
               head (the cases of the reference tests tests/test_data_loss.py:68-85, tests/test_gemma4.py:266-277,
               in bf16) (--only ce)
  hf_qwen_block.pt  transformers' own Qwen3_5MoeSparseMoeBlock (the module the reference's tests/test_moe.py:10-36
               pins moe_forward against) at the reference's tiny config (smel/tiny.py: hidden 256, 32 experts,
               top-4, expert and shared intermediate 64): weights, inputs, the fp32 and bf16 forward and the input
               gradients of an upstream gradient (--only hf; needs transformers' qwen3_5_moe module)
  dequant_torch.pt  smel/quant.py:87-94 dequant_int4_torch in bf16 (two roundings) of the quant.pt bank (--only
               dequant_torch)
  lora_fns.pt  smel/lora.py:61-83 lora_linear and lora_gate_up in fp32 on bf16-representable inputs: outputs and the
               gradients w.r.t. x, A and B of a seeded upstream gradient (--only lora)
  hf_gemma_block.pt  the MoE part of transformers' own Gemma4TextDecoderLayer after the attention residual (dense
               MLP, router, experts, the four feed-forward norms, layer_scalar, called in the order of the module's
               forward) at the reference's tiny Gemma 4 config (smel/tiny.py: hidden 256, 16 experts, top-4), fp32
               and bf16 forward and input gradients (--only hf_gemma; needs transformers' gemma4 module)
The test-suite never imports the reference; it only reads these files.
"""
import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def lora_tensors(H, I, S, n_sel, r, alpha, gen):
    """A: PEFT kaiming_uniform(a=sqrt(5)) bound 1/sqrt(in); B ~ N(0, 0.02) so the LoRA contributes."""
    def a(*s):
        return (torch.rand(*s, generator=gen) * 2 - 1) / (s[-1] ** 0.5)

    def b(*s):
        return torch.randn(*s, generator=gen) * 0.02

    ex = {"A_gate": a(n_sel, r, H), "B_gate": b(n_sel, I, r), "A_up": a(n_sel, r, H), "B_up": b(n_sel, I, r),
          "A_down": a(n_sel, r, I), "B_down": b(n_sel, H, r)}
    sh = {"A_gate": a(r, H), "B_gate": b(S, r), "A_up": a(r, H), "B_up": b(S, r), "A_down": a(r, S),
          "B_down": b(H, r)}
    return ex, sh


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SMEL_REFERENCE"),
                    help="the smel-ft source tree (default: $SMEL_REFERENCE)")
    ap.add_argument("--only", default=None, choices=[None, "pack", "ce", "hf", "hf_gemma", "dequant_torch", "lora"])
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference <smel-ft source tree> or set SMEL_REFERENCE")
    sys.path.insert(0, args.reference)
    if args.only == "pack":
        make_pack()
        return
    if args.only == "ce":
        make_ce()
        return
    if args.only == "hf":
        make_hf()
        return
    if args.only == "hf_gemma":
        make_hf_gemma()
        return
    if args.only == "dequant_torch":
        make_dequant_torch()
        return
    if args.only == "lora":
        make_lora_fns()
        return
    from smel.lora import ExpertsLoRA, LayerLoRA, MLPLoRA
    from smel.moe import FrozenExpertsFn, BF16Experts, Int4Experts, LayerExperts, moe_forward, route
    from smel.quant import dequant_int4_torch, quantize_int4

    torch.set_num_threads(4)

    # ------------------------------------------------------------------ quant
    g = torch.Generator().manual_seed(11)
    w = torch.randn(4, 96, 256, generator=g) * 0.02
    w[0, 0, :64] = 0.37  # a constant group (scale clamps to 1e-8)
    pk = quantize_int4(w, 64)
    deq = dequant_int4_torch(pk["q"], pk["scale"], pk["zero"], torch.float32)
    gq = torch.randint(0, 16, (4, 8, 128), generator=g)
    gs = (torch.rand(4, 8, 2, generator=g) + 0.5).bfloat16().float()
    gz = torch.randn(4, 8, 2, generator=g).bfloat16().float()
    grid = (gq.reshape(4, 8, 2, 64).float() * gs[..., None] + gz[..., None]).reshape(4, 8, 128)
    pg = quantize_int4(grid, 64)
    torch.save({"w": w, "q": pk["q"], "scale": pk["scale"], "zero": pk["zero"], "deq_f32": deq,
                "grid_w": grid, "grid_q": pg["q"], "grid_scale": pg["scale"], "grid_zero": pg["zero"],
                "grid_back": dequant_int4_torch(pg["q"], pg["scale"], pg["zero"], torch.float32)},
               os.path.join(HERE, "quant.pt"))

    # ------------------------------------------------------------------ dispatch (many ties)
    topi = torch.randint(0, 8, (97, 4), generator=g)
    topi[10:20] = 3
    flat = topi.reshape(-1)
    order = torch.argsort(flat, stable=True)
    torch.save({"topi": topi, "E": 8, "order": order, "tok": order // 4, "counts": torch.bincount(flat, minlength=8)},
               os.path.join(HERE, "dispatch.pt"))

    # ------------------------------------------------------------------ config 1 (tiny, fp32)
    H, E, K, I, S, T, r, alpha = 64, 8, 2, 64, 64, 128, 8, 16.0
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, H, generator=g)
    W = {"mlp.gate.weight": torch.randn(E, H, generator=g) * 0.02,
         "mlp.shared_expert.gate_proj.weight": torch.randn(S, H, generator=g) * 0.02,
         "mlp.shared_expert.up_proj.weight": torch.randn(S, H, generator=g) * 0.02,
         "mlp.shared_expert.down_proj.weight": torch.randn(H, S, generator=g) * 0.02,
         "mlp.shared_expert_gate.weight": torch.randn(1, H, generator=g) * 0.02}
    gu = torch.randn(E, 2 * I, H, generator=g) * 0.02
    dn = torch.randn(E, H, I, generator=g) * 0.02
    sel = [0, 1]
    exl, shl = lora_tensors(H, I, S, len(sel), r, alpha, g)
    gy = torch.randn(T, H, generator=g)
    bank = Int4Experts(quantize_int4(gu, 64), quantize_int4(dn, 64), dtype=torch.float32)

    def run(dtype):
        xd = x.to(dtype).clone().requires_grad_(True)
        Wd = {k: v.to(dtype) for k, v in W.items()}
        bank_d = Int4Experts(bank.gu, bank.dn, dtype=dtype)
        ex = LayerExperts(bank_d, sel, gu[sel].to(dtype).clone(), dn[sel].to(dtype).clone(), group=4)
        le = ExpertsLoRA(sel, H, I, r, alpha)
        ls = MLPLoRA(H, S, r, alpha)
        with torch.no_grad():
            for n, v in exl.items():
                getattr(le, n).copy_(v)
            for n, v in shl.items():
                getattr(ls, n).copy_(v)
        lora = LayerLoRA(le, ls)
        rec = {}
        out = moe_forward(xd, Wd, ex, K, lora, stats=lambda p, v, i: rec.update(probs=p.detach(), topv=v.detach(),
                                                                              topi=i.detach()))
        out.backward(gy.to(dtype))
        res = {"out": out.detach(), "dx": xd.grad.detach(), **rec}
        for n in exl:
            res["g_ex_" + n] = getattr(le, n).grad.detach().clone()
            res["g_sh_" + n] = getattr(ls, n).grad.detach().clone()
        return res

    res32 = run(torch.float32)
    flat = res32["topi"].reshape(-1)
    order = torch.argsort(flat, stable=True)
    torch.save({"cfg": dict(H=H, E=E, K=K, I=I, S=S, T=T, r=r, alpha=alpha, sel=sel, act="silu"),
                "x": x, "W": W, "gu": gu, "dn": dn, "gy": gy, "lora_ex": exl, "lora_sh": shl,
                "gu_q": bank.gu["q"], "gu_scale": bank.gu["scale"], "gu_zero": bank.gu["zero"],
                "dn_q": bank.dn["q"], "dn_scale": bank.dn["scale"], "dn_zero": bank.dn["zero"],
                "order": order, "counts": torch.bincount(flat, minlength=E), **res32},
               os.path.join(HERE, "moe_c1.pt"))
    res16 = run(torch.bfloat16)
    torch.save(res16, os.path.join(HERE, "moe_c1_bf16.pt"))

    # route alone on the config-1 inputs, fp32 (routing indices and weights)
    probs, topv, topi = route(x, W["mlp.gate.weight"], K)
    torch.save({"probs": probs, "topv": topv, "topi": topi}, os.path.join(HERE, "route_c1.pt"))

    # ------------------------------------------------------------------ frozen experts, GELU-tanh, empty expert
    g = torch.Generator().manual_seed(5)
    Ef, Hf, If, N = 6, 32, 24, 50
    fgu, fdn = torch.randn(Ef, 2 * If, Hf, generator=g) * 0.2, torch.randn(Ef, Hf, If, generator=g) * 0.2
    counts = [9, 0, 12, 7, 15, 7]
    xf = torch.randn(N, Hf, generator=g, dtype=torch.float64).float().requires_grad_(True)
    gyf = torch.randn(N, Hf, generator=g)
    yf = FrozenExpertsFn.apply(xf, counts, BF16Experts(fgu, fdn), 2, "gelu_tanh")
    yf.backward(gyf)
    torch.save({"gu": fgu, "dn": fdn, "counts": torch.tensor(counts), "x": xf.detach(), "gy": gyf, "y": yf.detach(),
                "dx": xf.grad.detach()}, os.path.join(HERE, "frozen_gelu.pt"))

    # ------------------------------------------------------------------ Gemma 4 MoE block (layer_runner.py:252-261)
    from smel.layer_runner import rmsnorm as ref_rmsnorm
    from smel.moe import mlp_lora, route_gemma4, routed_experts
    H, E, K, I, S, T, r, alpha, eps = 64, 8, 2, 64, 128, 96, 8, 16.0, 1e-6
    sel = [2, 5]
    g = torch.Generator().manual_seed(31)
    rn = lambda *sh, std=1.0: torch.randn(*sh, generator=g) * std  # noqa: E731
    W = {"router.scale": 1.0 + rn(H, std=0.2), "router.proj.weight": rn(E, H, std=0.3),
         "router.per_expert_scale": 0.5 + torch.rand(E, generator=g),
         "mlp.gate_proj.weight": rn(S, H, std=0.05), "mlp.up_proj.weight": rn(S, H, std=0.05),
         "mlp.down_proj.weight": rn(H, S, std=0.05),
         "post_feedforward_layernorm_1.weight": 1.0 + rn(H, std=0.1),
         "pre_feedforward_layernorm_2.weight": 1.0 + rn(H, std=0.1),
         "post_feedforward_layernorm_2.weight": 1.0 + rn(H, std=0.1),
         "post_feedforward_layernorm.weight": 1.0 + rn(H, std=0.1), "layer_scalar": torch.tensor([0.7])}
    gu, dn = rn(E, 2 * I, H, std=0.05), rn(E, H, I, std=0.05)
    qgu, qdn = quantize_int4(gu, 64), quantize_int4(dn, 64)
    ex = LayerExperts(Int4Experts(qgu, qdn, dtype=torch.float32), sel, gu[sel].clone(), dn[sel].clone(),
                      act="gelu_tanh")
    lex_t, lsh_t = lora_tensors(H, I, S, len(sel), r, alpha, g)
    lex_m, lsh_m = ExpertsLoRA(sel, H, I, r, alpha), MLPLoRA(H, S, r, alpha)
    with torch.no_grad():
        for n in ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down"):
            getattr(lex_m, n).copy_(lex_t[n])
            getattr(lsh_m, n).copy_(lsh_t[n])
    h, xm, gy = rn(T, H).requires_grad_(True), rn(T, H).requires_grad_(True), rn(T, H)
    m = mlp_lora(xm, W["mlp.gate_proj.weight"], W["mlp.up_proj.weight"], W["mlp.down_proj.weight"], lsh_m,
                 "gelu_tanh", None)
    m = ref_rmsnorm(m, W["post_feedforward_layernorm_1.weight"], eps, False)
    probs, topv, topi = route_gemma4(h, W, K, eps)
    e = routed_experts(ref_rmsnorm(h, W["pre_feedforward_layernorm_2.weight"], eps, False), topv, topi, ex, lex_m)
    e = ref_rmsnorm(e, W["post_feedforward_layernorm_2.weight"], eps, False)
    out = (h + ref_rmsnorm(m + e, W["post_feedforward_layernorm.weight"], eps, False)) * W["layer_scalar"]
    out.backward(gy)
    torch.save({"cfg": dict(H=H, E=E, K=K, I=I, S=S, T=T, r=r, alpha=alpha, eps=eps, sel=sel, act="gelu_tanh"),
                "W": W, "gu": gu, "dn": dn, "gu_q": qgu["q"], "gu_scale": qgu["scale"], "gu_zero": qgu["zero"],
                "dn_q": qdn["q"], "dn_scale": qdn["scale"], "dn_zero": qdn["zero"], "lora_ex": lex_t,
                "lora_sh": lsh_t, "h": h.detach(), "xm": xm.detach(), "gy": gy, "out": out.detach(),
                "probs": probs.detach(), "topv": topv.detach(), "topi": topi, "dh": h.grad, "dxm": xm.grad,
                "g_lora_ex": {n: getattr(lex_m, n).grad for n in lex_t},
                "g_lora_sh": {n: getattr(lsh_m, n).grad for n in lsh_t}}, os.path.join(HERE, "gemma_block.pt"))
    make_pack()
    print("golden fixtures written to", HERE)


def make_dequant_torch():
    """The reference's torch dequant in bf16 (quant.py:87-94: product and sum each rounded to bf16) of quant.pt."""
    from smel.quant import dequant_int4_torch
    d = torch.load(os.path.join(HERE, "quant.pt"), weights_only=False)
    out = {"bf16": dequant_int4_torch(d["q"], d["scale"], d["zero"], torch.bfloat16),
           "grid_bf16": dequant_int4_torch(d["grid_q"], d["grid_scale"], d["grid_zero"], torch.bfloat16)}
    torch.save(out, os.path.join(HERE, "dequant_torch.pt"))


def make_lora_fns():
    """lora_linear / lora_gate_up (smel/lora.py:61-83) in fp32 with autograd, inputs rounded to bf16 first so a bf16
    implementation sees the same values."""
    from smel.lora import lora_gate_up, lora_linear
    g = torch.Generator().manual_seed(21)
    T, Kd, N, I, r, s = 150, 256, 192, 128, 16, 2.0

    def bf(t):
        return t.bfloat16().float()

    x = bf(torch.randn(T, Kd, generator=g))
    w = bf(torch.randn(N, Kd, generator=g) * 0.05)
    A = (torch.rand(r, Kd, generator=g) * 2 - 1) / Kd ** 0.5
    B = torch.randn(N, r, generator=g) * 0.05
    gy = torch.randn(T, N, generator=g)
    xr, Ar, Br = x.clone().requires_grad_(True), A.clone().requires_grad_(True), B.clone().requires_grad_(True)
    y = lora_linear(xr, w, Ar, Br, s)
    y.backward(gy)
    lin = {"x": x, "w": w, "A": A, "B": B, "scale": s, "gy": gy, "y": y.detach(), "dx": xr.grad, "dA": Ar.grad,
           "dB": Br.grad}
    wgu = bf(torch.randn(2 * I, Kd, generator=g) * 0.05)
    pr = {n: ((torch.rand(r, Kd, generator=g) * 2 - 1) / Kd ** 0.5 if n.startswith("A") else
              torch.randn(I, r, generator=g) * 0.05) for n in ("A_gate", "B_gate", "A_up", "B_up")}
    gg, gu_ = torch.randn(T, I, generator=g), torch.randn(T, I, generator=g)
    xr = x.clone().requires_grad_(True)
    prr = {k: v.clone().requires_grad_(True) for k, v in pr.items()}
    gate, up = lora_gate_up(xr, wgu, prr["A_gate"], prr["B_gate"], prr["A_up"], prr["B_up"], s)
    (gate * gg + up * gu_).sum().backward()
    gu = {"x": x, "w": wgu, **pr, "scale": s, "g_gate": gg, "g_up": gu_, "gate": gate.detach(), "up": up.detach(),
          "dx": xr.grad, **{"d" + k: v.grad for k, v in prr.items()}}
    torch.save({"linear": lin, "gate_up": gu}, os.path.join(HERE, "lora_fns.pt"))


def make_pack():
    from smel.lora import ExpertsLoRA, MLPLoRA
    from smel.pack import merge_experts, merge_mlp, pack_layer
    g = torch.Generator().manual_seed(21)
    E, H, I, S, r = 6, 128, 64, 64, 8
    t = {"mlp.gate.weight": torch.randn(E, H, generator=g) * 0.05,
         "mlp.shared_expert.gate_proj.weight": torch.randn(S, H, generator=g) * 0.02,
         "mlp.shared_expert.up_proj.weight": torch.randn(S, H, generator=g) * 0.02,
         "mlp.shared_expert.down_proj.weight": torch.randn(H, S, generator=g) * 0.02,
         "linear_attn.A_log": torch.randn(4, generator=g),
         "step.count": torch.arange(3, dtype=torch.int64),
         "mlp.experts.gate_up_proj": torch.randn(E, 2 * I, H, generator=g) * 0.02,
         "mlp.experts.down_proj": torch.randn(E, H, I, generator=g) * 0.02}
    sel = [4, 1]
    packed = pack_layer(t, sel, 64)
    lex = ExpertsLoRA(sel, H, I, r, 16.0)
    lsh = MLPLoRA(H, S, r, 16.0)
    with torch.no_grad():
        for m in (lex, lsh):
            for n in ("B_gate", "B_up", "B_down"):
                getattr(m, n).copy_(torch.randn(getattr(m, n).shape, generator=g) * 0.05)
    mgu, mdn = merge_experts(t["mlp.experts.gate_up_proj"].bfloat16(), t["mlp.experts.down_proj"].bfloat16(), lex)
    mg, mu, md = merge_mlp(t["mlp.shared_expert.gate_proj.weight"].bfloat16(),
                           t["mlp.shared_expert.up_proj.weight"].bfloat16(),
                           t["mlp.shared_expert.down_proj.weight"].bfloat16(), lsh)
    torch.save({"t": t, "sel": sel, "packed": packed,
                "lora_ex": {n: p.detach().clone() for n, p in lex.named_parameters()},
                "lora_sh": {n: p.detach().clone() for n, p in lsh.named_parameters()}, "r": r, "alpha": 16.0,
                "merged_gu": mgu, "merged_dn": mdn, "merged_mlp": (mg, mu, md)}, os.path.join(HERE, "pack.pt"))


def make_ce():
    from smel.loss import LMHead, chunked_ce
    torch.set_num_threads(4)
    g = torch.Generator().manual_seed(31)
    cases = {}
    # bf16 head, ragged last vocabulary chunk (952 rows) and token chunk (8 rows)
    V, H, N = 3000, 128, 200
    W = (torch.randn(V, H, generator=g) * 0.05).bfloat16()
    h = torch.randn(N, H, generator=g).bfloat16()
    tgt = torch.randint(0, V, (N,), generator=g)
    for name, int8 in (("bf16", False), ("int8", True)):
        head = LMHead.from_weight(W, int8=int8, vocab_chunk=1024)
        hh = h.clone().requires_grad_(True)
        loss = chunked_ce(hh, head, tgt, denom=N, token_chunk=64)
        loss.backward()
        c = {"h": h, "tgt": tgt, "V": V, "vocab_chunk": 1024, "token_chunk": 64, "softcap": 0.0, "denom": float(N),
             "loss": loss.detach(), "grad": hh.grad.clone()}
        if int8:
            c["q"], c["scale"] = head.q["q"], head.q["scale"]
        else:
            c["w"] = W
        cases[name] = c
    # softcapped head (Gemma), logits well into the cap's curve
    V, H, N = 3000, 64, 120
    W = (torch.randn(V, H, generator=g) * 0.5).bfloat16()
    h = (torch.randn(N, H, generator=g) * 3).bfloat16()
    tgt = torch.randint(0, V, (N,), generator=g)
    head = LMHead.from_weight(W, vocab_chunk=700, softcap=30.0)
    hh = h.clone().requires_grad_(True)
    loss = chunked_ce(hh, head, tgt, denom=N, token_chunk=50)
    loss.backward()
    cases["softcap"] = {"h": h, "tgt": tgt, "w": W, "V": V, "vocab_chunk": 700, "token_chunk": 50, "softcap": 30.0,
                        "denom": float(N), "loss": loss.detach(), "grad": hh.grad.clone()}
    # the loss alone (need_grad=False path)
    with torch.no_grad():
        cases["softcap"]["loss_nograd"] = chunked_ce(h, head, tgt, denom=N, token_chunk=50, need_grad=False)
    torch.save(cases, os.path.join(HERE, "ce.pt"))


def make_hf():
    from smel.tiny import tiny_text_config
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock
    torch.set_num_threads(4)
    torch.manual_seed(0)
    cfg = tiny_text_config()
    cfg._experts_implementation = "eager"  # the plain per-expert loop of the module (no kernel dispatch)
    blk = Qwen3_5MoeSparseMoeBlock(cfg).eval()
    g = torch.Generator().manual_seed(41)
    with torch.no_grad():
        for n, p in blk.named_parameters():
            # as smel/tiny.py build_tiny_model: a non-trivial router, experts N(0, 0.05); shared expert likewise.
            # Values are rounded to bf16 so that the fixture stores them in bf16 and the fp32 run sees the same ones.
            p.copy_((torch.randn(p.shape, generator=g) * (0.3 if n == "gate.weight" else 0.05)).bfloat16().float())
    T, H = 256, blk.gate.weight.shape[1]
    x = torch.randn(T, H, generator=g).bfloat16().float()
    gy = torch.randn(T, H, generator=g).bfloat16().float()
    out = {}
    for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        b = blk.to(dt)
        xx = x.to(dt).detach().clone().requires_grad_(True)
        y = b(xx[None])
        y = (y[0] if isinstance(y, tuple) else y)[0]
        y.backward(gy.to(dt))
        out[name] = (y.detach().clone(), xx.grad.detach().clone())
    blk = blk.float()
    torch.save({"W": {"mlp." + k: v.detach().bfloat16() for k, v in blk.state_dict().items()}, "x": x.bfloat16(),
                "gy": gy.bfloat16(),
                "top_k": 4, "sel": [0, 3, 7, 30], "out_fp32": out["fp32"][0], "dx_fp32": out["fp32"][1],
                "out_bf16": out["bf16"][0], "dx_bf16": out["bf16"][1]}, os.path.join(HERE, "hf_qwen_block.pt"))


def make_hf_gemma():
    from smel.tiny import tiny_gemma4_config
    from transformers.models.gemma4.modeling_gemma4 import Gemma4TextDecoderLayer
    torch.set_num_threads(4)
    torch.manual_seed(0)
    cfg = tiny_gemma4_config()
    cfg._experts_implementation = "eager"  # the plain per-expert loop of the module
    cfg._attn_implementation = "sdpa"
    layer = Gemma4TextDecoderLayer(cfg, layer_idx=0).eval()
    g = torch.Generator().manual_seed(43)
    with torch.no_grad():
        for n, p in layer.named_parameters():
            if n.startswith("self_attn"):
                continue
            # as smel/tiny.py build_tiny_gemma4: non-trivial norms and scales (Gemma norms multiply by w directly)
            if n.endswith("norm.weight") or n.endswith("layernorm.weight") or n.endswith("router.scale"):
                v = torch.randn(p.shape, generator=g) * 0.2 + 1.0
            elif n.endswith("per_expert_scale"):
                v = torch.rand(p.shape, generator=g) + 0.5
            elif n.endswith("router.proj.weight"):
                v = torch.randn(p.shape, generator=g) * 0.3
            else:
                v = torch.randn(p.shape, generator=g) * 0.05
            p.copy_(v.bfloat16().float())  # bf16-exact, so the fixture stores bf16 and the fp32 run sees the same
        layer.layer_scalar.fill_(0.875)
    T, H = 256, cfg.hidden_size
    h = torch.randn(T, H, generator=g).bfloat16().float()
    gy = torch.randn(T, H, generator=g).bfloat16().float()

    def block(L, hh):
        # the MoE part of Gemma4TextDecoderLayer.forward, after `residual = hidden_states` (attention residual)
        m = L.post_feedforward_layernorm_1(L.mlp(L.pre_feedforward_layernorm(hh)))
        _, w, idx = L.router(hh)
        e = L.post_feedforward_layernorm_2(L.experts(L.pre_feedforward_layernorm_2(hh), idx, w))
        return (hh + L.post_feedforward_layernorm(m + e)) * L.layer_scalar, idx

    out = {}
    for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        L = layer.to(dt)
        hh = h.to(dt).detach().clone().requires_grad_(True)
        y, idx = block(L, hh)
        y.backward(gy.to(dt))
        out[name] = (y.detach().clone(), hh.grad.detach().clone(), idx.clone())
    layer = layer.float()
    W = {k: v.detach().bfloat16() for k, v in layer.state_dict().items() if not k.startswith("self_attn")}
    torch.save({"W": W, "h": h.bfloat16(), "gy": gy.bfloat16(), "top_k": cfg.top_k_experts,
                "eps": cfg.rms_norm_eps, "out_fp32": out["fp32"][0], "dh_fp32": out["fp32"][1],
                "topi_fp32": out["fp32"][2], "out_bf16": out["bf16"][0], "dh_bf16": out["bf16"][1]},
               os.path.join(HERE, "hf_gemma_block.pt"))


if __name__ == "__main__":
    main()
