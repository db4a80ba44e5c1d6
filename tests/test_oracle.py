"""The CPU oracle against golden vectors produced by the reference implementation (tests/golden/make_golden.py)."""
import numpy as np
import torch

from oracle import moe_oracle as O


def test_quantize_matches_reference_bit_exact(golden):
    d = golden("quant.pt")
    pk = O.quantize_int4(d["w"], 64)
    assert torch.equal(pk["q"], d["q"])
    assert torch.equal(pk["scale"].view(torch.int16), d["scale"].view(torch.int16))
    assert torch.equal(pk["zero"].view(torch.int16), d["zero"].view(torch.int16))


def test_dequant_fp32_matches_reference_bit_exact(golden):
    d = golden("quant.pt")
    w = O.dequant_int4(d["q"], d["scale"], d["zero"], torch.float32)
    assert torch.equal(w, d["deq_f32"])


def test_int4_roundtrip_on_grid(golden):
    """Known answer (reference tests/test_quant_merge.py:14-23): on-grid weights survive quantize -> dequant up to
    the bf16 rounding of scale/zero."""
    d = golden("quant.pt")
    pk = O.quantize_int4(d["grid_w"], 64)
    assert torch.equal(pk["q"], d["grid_q"])
    back = O.dequant_int4(pk["q"], pk["scale"], pk["zero"])
    assert torch.equal(back, d["grid_back"])
    assert O.rel_err(back, d["grid_w"]) < 5e-3


def test_nibble_order_low_is_even_column():
    codes = np.arange(16, dtype=np.uint8).reshape(1, 16)
    q = O.pack_nibbles(codes)
    assert q.tolist() == [[0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE]]
    assert np.array_equal(O.unpack_nibbles(q), codes)


def test_dispatch_matches_reference(golden):
    d = golden("dispatch.pt")
    order, tok, counts = O.dispatch(d["topi"].numpy(), d["E"])
    assert np.array_equal(order, d["order"].numpy())
    assert np.array_equal(tok, d["tok"].numpy())
    assert np.array_equal(counts, d["counts"].numpy())


def test_dispatch_padded_layout(golden):
    d = golden("dispatch.pt")
    topi = d["topi"].numpy()
    sel = np.zeros(8, dtype=np.uint8)
    sel[[3, 5]] = 1
    counts, gcounts, offsets, row_of, src_of = O.dispatch_padded(topi, 8, sel, pad=64)
    assert np.array_equal(counts, d["counts"].numpy())
    assert all(gcounts[e] % 64 == 0 for e in (3, 5))
    # the unpadded rank order is the reference's stable argsort
    order, _, _ = O.dispatch(topi, 8)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    for j, i in enumerate(order):
        e = topi.reshape(-1)[i]
        assert row_of[i] - offsets[e] == j - starts[e]
    assert (src_of[row_of] == np.arange(row_of.size)).all()
    assert (src_of == -1).sum() == int((gcounts - counts).sum())


def test_route_matches_reference(golden):
    d = golden("moe_c1.pt")
    r = golden("route_c1.pt")
    probs, topv, topi = O.route(d["x"], d["W"]["mlp.gate.weight"], d["cfg"]["K"])
    assert torch.allclose(probs, r["probs"], rtol=0, atol=1e-7)
    # no ties at this seed: indices must match exactly
    assert torch.equal(topi, r["topi"])
    assert torch.allclose(topv, r["topv"], rtol=0, atol=1e-6)


def _c1_oracle(d, dtype=torch.float64):
    cfg = d["cfg"]
    gu = O.dequant_int4(d["gu_q"], d["gu_scale"], d["gu_zero"]).to(dtype)
    dn = O.dequant_int4(d["dn_q"], d["dn_scale"], d["dn_zero"]).to(dtype)
    x = d["x"].to(dtype).requires_grad_(True)
    W = {k: v.to(dtype) for k, v in d["W"].items()}
    sel = cfg["sel"]
    lex = {k: v.to(dtype).requires_grad_(True) for k, v in d["lora_ex"].items()}
    lsh = {k: v.to(dtype).requires_grad_(True) for k, v in d["lora_sh"].items()}
    scale = cfg["alpha"] / cfg["r"]
    out, probs, topv, topi = O.moe_layer(x, W, gu, dn, cfg["K"], sel, d["gu"][sel].to(dtype), d["dn"][sel].to(dtype),
                                         {**lex, "scale": scale}, {**lsh, "scale": scale}, topi=d["topi"])
    out.backward(d["gy"].to(dtype))
    return out, x.grad, lex, lsh, topv


def test_moe_forward_backward_matches_reference_fp32(golden):
    """Config 1: the oracle (fp64) reproduces the reference's fp32 output, dX and all LoRA gradients."""
    d = golden("moe_c1.pt")
    out, dx, lex, lsh, topv = _c1_oracle(d)
    assert O.rel_err(out, d["out"]) < 1e-5
    assert O.rel_err(dx, d["dx"]) < 1e-5
    assert O.rel_err(topv, d["topv"]) < 1e-6
    for n in lex:
        assert O.rel_err(lex[n].grad, d["g_ex_" + n]) < 1e-5, n
        assert O.rel_err(lsh[n].grad, d["g_sh_" + n]) < 1e-5, n


def test_frozen_experts_gelu_backward_matches_reference(golden):
    d = golden("frozen_gelu.pt")
    x = d["x"].double().requires_grad_(True)
    y = O.frozen_experts(x, d["counts"].tolist(), d["gu"].double(), d["dn"].double(), "gelu_tanh")
    assert O.rel_err(y, d["y"]) < 1e-5
    y.backward(d["gy"].double())
    assert O.rel_err(x.grad, d["dx"]) < 1e-5
    manual = O.frozen_experts_backward(d["x"].double(), d["gy"].double(), d["counts"].tolist(), d["gu"].double(),
                                       d["dn"].double(), "gelu_tanh")
    assert O.rel_err(manual, d["dx"]) < 1e-5


def _gemma_oracle(d, dt=torch.float32, topi=None, h=None, xm=None):
    c = d["cfg"]
    gu = O.dequant_int4(d["gu_q"], d["gu_scale"], d["gu_zero"], dt)
    dn = O.dequant_int4(d["dn_q"], d["dn_scale"], d["dn_zero"], dt)
    s = c["alpha"] / c["r"]
    lex = {k: v.to(dt).clone().requires_grad_(True) for k, v in d["lora_ex"].items()}
    lsh = {k: v.to(dt).clone().requires_grad_(True) for k, v in d["lora_sh"].items()}
    h = (d["h"] if h is None else h).to(dt).clone().requires_grad_(True)
    xm = (d["xm"] if xm is None else xm).to(dt).clone().requires_grad_(True)
    W = {k: v.to(dt) for k, v in d["W"].items()}
    out, probs, topv, topi = O.moe_block_gemma4(h, xm, W, gu, dn, c["K"], c["eps"], c["sel"], d["gu"][c["sel"]].to(dt),
                                                d["dn"][c["sel"]].to(dt), {**lex, "scale": s}, {**lsh, "scale": s},
                                                c["act"], topi)
    return out, probs, topv, topi, h, xm, lex, lsh


def test_gemma_block_matches_reference_fp32(golden):
    """route_gemma4 + the Gemma 4 MoE block (smel/layer_runner.py:252-261) against the reference's own fp32 run."""
    d = golden("gemma_block.pt")
    out, probs, topv, topi, h, xm, lex, lsh = _gemma_oracle(d)
    assert torch.equal(topi, d["topi"])
    assert O.rel_err(probs, d["probs"]) < 1e-6 and O.rel_err(topv, d["topv"]) < 1e-6
    assert O.rel_err(out, d["out"]) < 1e-5
    out.backward(d["gy"])
    assert O.rel_err(h.grad, d["dh"]) < 1e-5 and O.rel_err(xm.grad, d["dxm"]) < 1e-5
    for n in lex:
        assert O.rel_err(lex[n].grad, d["g_lora_ex"][n]) < 1e-5, n
        assert O.rel_err(lsh[n].grad, d["g_lora_sh"][n]) < 1e-5, n


def test_rmsnorm_oracle_forms():
    """The three weight modes of smel/layer_runner.py:110-121 and the fused add of :124-130."""
    g = torch.Generator().manual_seed(3)
    x, h, w = torch.randn(7, 64, generator=g), torch.randn(7, 64, generator=g), torch.randn(64, generator=g)
    rstd = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert torch.allclose(O.rmsnorm(x, w, 1e-6, True), x * rstd * (1 + w), atol=1e-6)
    assert torch.allclose(O.rmsnorm(x, w, 1e-6, False), x * rstd * w, atol=1e-6)
    assert torch.allclose(O.rmsnorm(x, None, 1e-6, False), x * rstd, atol=1e-6)
    s, y = O.add_rmsnorm(h, x, w, 1e-6, False)
    assert torch.equal(s, h + x) and torch.allclose(y, O.rmsnorm(h + x, w, 1e-6, False))


def test_oracle_dequant_stepwise_equals_reference(golden):
    """dequant_int4_torch in bf16 (two roundings) as the reference computes it (tests/golden/dequant_torch.pt)."""
    d, t = golden("quant.pt"), golden("dequant_torch.pt")
    a = O.dequant_int4_stepwise(d["q"], d["scale"], d["zero"], torch.bfloat16)
    assert torch.equal(a.view(torch.int16), t["bf16"].view(torch.int16))
    b = O.dequant_int4_stepwise(d["grid_q"], d["grid_scale"], d["grid_zero"], torch.bfloat16)
    assert torch.equal(b.view(torch.int16), t["grid_bf16"].view(torch.int16))
    # and it is a different function from the single-rounding dequant on a large share of the weights
    single = O.dequant_int4(d["q"], d["scale"], d["zero"]).to(torch.bfloat16)
    assert (single.view(torch.int16) != a.view(torch.int16)).float().mean() > 0.2


def test_oracle_lora_functions_equal_reference(golden):
    """lora_linear / lora_gate_up of the oracle against the reference's own fp32 outputs and gradients."""
    d = golden("lora_fns.pt")
    L = d["linear"]
    x, A, B = (L[k].clone().requires_grad_(True) for k in ("x", "A", "B"))
    y = O.lora_linear(x, L["w"], A, B, L["scale"])
    y.backward(L["gy"])
    for name, a, b in (("y", y, L["y"]), ("dx", x.grad, L["dx"]), ("dA", A.grad, L["dA"]), ("dB", B.grad, L["dB"])):
        assert O.rel_err(a, b) < 1e-5, name
    G = d["gate_up"]
    x = G["x"].clone().requires_grad_(True)
    p = {k: G[k].clone().requires_grad_(True) for k in ("A_gate", "B_gate", "A_up", "B_up")}
    g, u = O.lora_gate_up(x, G["w"], p["A_gate"], p["B_gate"], p["A_up"], p["B_up"], G["scale"])
    (g * G["g_gate"] + u * G["g_up"]).sum().backward()
    assert O.rel_err(g, G["gate"]) < 1e-5 and O.rel_err(u, G["up"]) < 1e-5
    assert O.rel_err(x.grad, G["dx"]) < 1e-5
    for k in p:
        assert O.rel_err(p[k].grad, G["d" + k]) < 1e-5, k
