"""GPU checks of the drop-in boundary pieces beyond the layer call: the reference's dequant_int4_torch rounding
(smel/quant.py:87-94), lora_linear / lora_gate_up (smel/lora.py:61-83) on the GEMM engine, FrozenExpertsFn over a
BF16Experts bank (smel/moe.py:18-32, 110-143), and the reference's activation-memory contract
(set_save_preactivations(False): the backward recomputes the gate/up pre-activations). Tolerances: bit-exact for the
dequant; max relative error 2e-2 and cosine 0.9999 against the reference's fp32 results for the bf16 GEMMs;
bit-identical results between the two activation-memory modes (the recompute runs the same tiles)."""
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

REL, COS = 2e-2, 0.9999


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    return torch.device("cuda:0")


def close(a, b, what, rel=REL, cos=COS):
    e, c = O.rel_err(a.float().cpu(), b.float().cpu()), O.cosine(a.float().cpu(), b.float().cpu())
    assert e <= rel and c >= cos, f"{what}: rel err {e:.3e}, cosine {c:.6f}"


def test_dequant_int4_torch_keeps_reference_rounding(dev, golden):
    import smelb
    d, t = golden("quant.pt"), golden("dequant_torch.pt")
    a = smelb.dequant_int4_torch(d["q"].to(dev), d["scale"].to(dev), d["zero"].to(dev), torch.bfloat16).cpu()
    assert torch.equal(a.view(torch.int16), t["bf16"].view(torch.int16))
    b = smelb.dequant_int4_torch(d["grid_q"].to(dev), d["grid_scale"].to(dev), d["grid_zero"].to(dev),
                                 torch.bfloat16).cpu()
    assert torch.equal(b.view(torch.int16), t["grid_bf16"].view(torch.int16))
    f32 = smelb.dequant_int4_torch(d["q"].to(dev), d["scale"].to(dev), d["zero"].to(dev), torch.float32).cpu()
    assert torch.equal(f32, d["deq_f32"])
    assert smelb.read_status() == 0


def test_lora_linear_vs_reference(dev, golden):
    import smelb
    L = golden("lora_fns.pt")["linear"]
    x = L["x"].bfloat16().to(dev).requires_grad_(True)
    A = L["A"].to(dev).requires_grad_(True)
    B = L["B"].to(dev).requires_grad_(True)
    y = smelb.lora_linear(x, L["w"].bfloat16().to(dev), A, B, L["scale"])
    y.backward(L["gy"].bfloat16().to(dev))
    close(y, L["y"], "y")
    close(x.grad, L["dx"], "dx")
    close(A.grad, L["dA"], "dA")
    close(B.grad, L["dB"], "dB")
    assert A.grad.dtype == torch.float32 and B.grad.dtype == torch.float32
    # leading dimensions are kept (the reference's non-2-D branch), and A = None is the plain projection
    y3 = smelb.lora_linear(x.detach().reshape(3, 50, -1), L["w"].bfloat16().to(dev), A.detach(), B.detach(),
                           L["scale"])
    assert y3.shape == (3, 50, y.shape[-1]) and torch.equal(y3.reshape(y.shape), y.detach())
    y0 = smelb.lora_linear(x.detach(), L["w"].bfloat16().to(dev), None, None, L["scale"])
    close(y0, L["x"] @ L["w"].t(), "plain projection")
    assert smelb.read_status() == 0


def test_lora_gate_up_vs_reference(dev, golden):
    import smelb
    G = golden("lora_fns.pt")["gate_up"]
    x = G["x"].bfloat16().to(dev).requires_grad_(True)
    p = {k: G[k].to(dev).requires_grad_(True) for k in ("A_gate", "B_gate", "A_up", "B_up")}
    g, u = smelb.lora_gate_up(x, G["w"].bfloat16().to(dev), p["A_gate"], p["B_gate"], p["A_up"], p["B_up"],
                              G["scale"])
    (g.float() * G["g_gate"].to(dev) + u.float() * G["g_up"].to(dev)).sum().backward()
    close(g, G["gate"], "gate")
    close(u, G["up"], "up")
    close(x.grad, G["dx"], "dx")
    for k in p:
        close(p[k].grad, G["d" + k], "d" + k)
    assert smelb.read_status() == 0


def test_lora_rank_must_be_multiple_of_8(dev):
    import smelb
    x = torch.randn(16, 128, device=dev).bfloat16()
    w = torch.randn(128, 128, device=dev).bfloat16()
    with pytest.raises(smelb.SmelbError, match="multiple of 8"):
        smelb.lora_linear(x, w, torch.randn(4, 128, device=dev), torch.randn(128, 4, device=dev), 2.0)


def test_frozen_experts_fn_bf16_bank(dev):
    import smelb
    g = torch.Generator(device=dev).manual_seed(7)
    E, H, I = 6, 256, 128
    counts = [40, 0, 130, 3, 64, 17]
    gu = (torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.05).bfloat16()
    dn = (torch.randn(E, H, I, generator=g, device=dev) * 0.05).bfloat16()
    xs = torch.randn(sum(counts), H, generator=g, device=dev).bfloat16().requires_grad_(True)
    gy = torch.randn(sum(counts), H, generator=g, device=dev).bfloat16()
    for act in ("silu", "gelu_tanh"):
        xs.grad = None
        y = smelb.FrozenExpertsFn.apply(xs, counts, smelb.BF16Experts(gu, dn), 32, act)
        y.backward(gy)
        x64 = xs.detach().cpu().double()
        close(y, O.frozen_experts(x64, counts, gu.cpu().double(), dn.cpu().double(), act), f"bf16 bank out {act}")
        close(xs.grad, O.frozen_experts_backward(x64, gy.cpu().double(), counts, gu.cpu().double(),
                                                 dn.cpu().double(), act), f"bf16 bank dx {act}")
    assert smelb.read_status() == 0


def test_save_preactivations_off_is_bit_identical(dev):
    """The reference's memory contract (only the inputs kept, pre-activations recomputed in the backward) gives the
    same bits as the default (pre-activations kept), for FrozenExpertsFn and for the whole layer with LoRA."""
    import smelb
    from smelb.synth import qwen_layer
    L = qwen_layer(T=300, H=256, E=16, K=4, I=128, S=128, n_sel=3, r=8, alpha=16.0, seed=8, device=dev)
    gy = torch.randn(L["x"].shape, generator=torch.Generator(device=dev).manual_seed(2), device=dev).bfloat16()
    params = list(L["lora"].parameters())

    def run():
        for p in params:
            p.grad = None
        x = L["x"].clone().requires_grad_(True)
        out = smelb.moe_forward(x, L["W"], L["ex"], 4, L["lora"])
        out.backward(gy)
        return out.detach(), x.grad, [p.grad.clone() for p in params]

    bank = L["ex"].frozen
    counts = [5, 0, 77, 31]
    xs = torch.randn(sum(counts), 256, device=dev).bfloat16()

    def run_frozen():
        x = xs.clone().requires_grad_(True)
        y = smelb.FrozenExpertsFn.apply(x, counts, smelb.Int4Experts(
            {k: v[:4] for k, v in bank.gu.items()}, {k: v[:4] for k, v in bank.dn.items()}), 32, "silu")
        y.backward(gy[:sum(counts)])
        return y.detach(), x.grad

    try:
        a, fa = run(), run_frozen()
        smelb.set_save_preactivations(False)
        b, fb = run(), run_frozen()
    finally:
        smelb.set_save_preactivations(True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    for ga, gb in zip(a[2], b[2]):
        assert torch.equal(ga, gb)
    assert torch.equal(fa[0], fb[0]) and torch.equal(fa[1], fb[1])
    assert smelb.read_status() == 0
