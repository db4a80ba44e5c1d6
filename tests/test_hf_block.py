"""The MoE block against transformers' own Qwen3_5MoeSparseMoeBlock, the module the reference pins its moe_forward
against (smel-ft tests/test_moe.py:10-36), at the reference's tiny config (hidden 256, 32 experts, top-4, expert and
shared intermediate 64). tests/golden/hf_qwen_block.pt holds the module's weights (bf16-exact), an input, an upstream
gradient and the module's fp32 and bf16 outputs and input gradients (tests/golden/make_golden.py --only hf).

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
