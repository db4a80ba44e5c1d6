"""The MoE block against transformers' own Qwen3_5MoeSparseMoeBlock, the module the reference pins its moe_forward
against (smel-ft tests/test_moe.py:10-36), at the reference's tiny config (hidden 256, 32 experts, top-4, expert and
shared intermediate 64). tests/golden/hf_qwen_block.pt holds the module's weights (bf16-exact), an input, an upstream
gradient and the module's fp32 and bf16 outputs and input gradients (tests/golden/make_golden.py --only hf).
tests/golden/hf_gemma_block.pt does the same for the MoE part of transformers' Gemma4TextDecoderLayer at the
reference's tiny Gemma 4 config (--only hf_gemma), against which smelb.moe_block_gemma4 is checked with the
reference's own bf16 bar (smel-ft tests/test_gemma4.py:123-133: error against HF fp32 at most 1.25 x HF bf16's
own error + 1e-2).

CPU: the oracle (oracle/moe_oracle.py) in fp32 equals the HF fp32 output within the reference test's fp32 bar (1e-5)
and its dX as well. GPU: smelb.moe_forward (bf16 compute) against the HF bf16 run within the reference test's bf16
bar (2e-2 relative error), with and without selected experts, forward and dX; also against HF fp32 (2e-2)."""
import pytest
import torch

from oracle import moe_oracle as O


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_oracle_matches_hf_block_fp32(golden):
    d = golden("hf_qwen_block.pt")
    W = {k: v.float() for k, v in d["W"].items()}
    x = d["x"].float().requires_grad_(True)
    out, _, _, _ = O.moe_layer(x, W, W["mlp.experts.gate_up_proj"], W["mlp.experts.down_proj"], d["top_k"])
    out.backward(d["gy"].float())
    assert _rel(out.detach(), d["out_fp32"]) < 1e-5
    assert _rel(x.grad, d["dx_fp32"]) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("with_sel", [False, True])
def test_moe_forward_matches_hf_block(golden, with_sel):
    import smelb
    d = golden("hf_qwen_block.pt")
    dev = torch.device("cuda", 0)
    W = {k: v.to(dev) for k, v in d["W"].items()}
    gu, dn = W.pop("mlp.experts.gate_up_proj"), W.pop("mlp.experts.down_proj")
    bank = smelb.BF16Experts(gu, dn)
    if with_sel:
        ids = torch.as_tensor(d["sel"], device=dev)
        ex = smelb.LayerExperts(bank, d["sel"], gu[ids].clone(), dn[ids].clone())
    else:
        ex = smelb.LayerExperts(bank)
    x = d["x"].to(dev).requires_grad_(True)
    out = smelb.moe_forward(x, W, ex, d["top_k"])
    out.backward(d["gy"].to(dev))
    for ref_out, ref_dx in ((d["out_bf16"], d["dx_bf16"]), (d["out_fp32"], d["dx_fp32"])):
        assert _rel(out.detach(), ref_out) < 2e-2, _rel(out.detach(), ref_out)
        assert _rel(x.grad, ref_dx) < 2e-2, _rel(x.grad, ref_dx)


@pytest.mark.gpu
def test_int4_bank_close_to_hf_block(golden):
    """The same block with its experts packed int4 group-64 (the format the reference trains with): the output moves
    by the quantization error only (the reference's own int4-vs-bf16 MoE bar, smel-ft
    tests/test_quant_merge.py:53-78, is 0.15)."""
    import smelb
    d = golden("hf_qwen_block.pt")
    dev = torch.device("cuda", 0)
    W = {k: v.to(dev) for k, v in d["W"].items()}
    gu, dn = W.pop("mlp.experts.gate_up_proj"), W.pop("mlp.experts.down_proj")
    ex = smelb.LayerExperts(smelb.Int4Experts.from_bf16(gu, dn))
    with torch.no_grad():
        out = smelb.moe_forward(d["x"].to(dev), W, ex, d["top_k"])
    assert _rel(out, d["out_fp32"]) < 0.15, _rel(out, d["out_fp32"])


# ------------------------------------------------------------------------------------------------------ Gemma 4
def _gemma_w(d, dtype, dev="cpu"):
    return {k: v.to(device=dev, dtype=dtype) for k, v in d["W"].items()}


def test_oracle_matches_hf_gemma_block_fp32(golden):
    d = golden("hf_gemma_block.pt")
    W = _gemma_w(d, torch.float32)
    h = d["h"].float().requires_grad_(True)
    xm = O.rmsnorm(h, W["pre_feedforward_layernorm.weight"], d["eps"], False)
    out, _, _, topi = O.moe_block_gemma4(h, xm, W, W["experts.gate_up_proj"], W["experts.down_proj"], d["top_k"],
                                         d["eps"])
    out.backward(d["gy"].float())
    assert torch.equal(topi, d["topi_fp32"])
    assert _rel(out.detach(), d["out_fp32"]) < 1e-4
    assert _rel(h.grad, d["dh_fp32"]) < 1e-4


@pytest.mark.gpu
def test_moe_block_gemma4_matches_hf(golden):
    import smelb
    d = golden("hf_gemma_block.pt")
    dev = torch.device("cuda", 0)
    W = _gemma_w(d, torch.bfloat16, dev)
    ex = smelb.LayerExperts(smelb.BF16Experts(W["experts.gate_up_proj"], W["experts.down_proj"]), act="gelu_tanh")
    h = d["h"].to(dev).requires_grad_(True)
    xm = smelb.rmsnorm(h, W["pre_feedforward_layernorm.weight"], d["eps"], False)
    out = smelb.moe_block_gemma4(h, xm, W, ex, d["top_k"], d["eps"], "gelu_tanh")
    out.backward(d["gy"].to(dev))
    for ours, hf16, hf32 in ((out.detach(), d["out_bf16"], d["out_fp32"]), (h.grad, d["dh_bf16"], d["dh_fp32"])):
        e_ours, e_hf = _rel(ours, hf32), _rel(hf16, hf32)
        assert e_ours < 1.25 * e_hf + 1e-2, (e_ours, e_hf)
