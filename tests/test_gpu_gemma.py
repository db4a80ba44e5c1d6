"""Row norms (smelb.norm) and the Gemma 4 path (route_gemma4, moe_block_gemma4) on the GPU against the oracle and
the reference's golden vectors (tests/golden/gemma_block.pt)."""
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    return torch.device("cuda:0")


def close(a, b, what, rel=2e-2, cos=0.9999):
    e, c = O.rel_err(a.float().cpu(), b.float().cpu()), O.cosine(a.float().cpu(), b.float().cpu())
    assert e <= rel and c >= cos, f"{what}: rel err {e:.3e}, cosine {c:.6f}"


@pytest.mark.parametrize("rows,C", [(37, 64), (300, 2048), (129, 2816)])
@pytest.mark.parametrize("mode", ["plus_one", "w", "none", "add"])
def test_rmsnorm_kernels_vs_oracle(dev, rows, C, mode):
    """Forward within 2 bf16 ulp of the fp32 torch form (smel/layer_runner.py:110-130) on the same bf16 inputs,
    backward within the tolerance of the other tests."""
    import smelb
    g = torch.Generator(device=dev).manual_seed(rows + C)
    x = torch.randn(rows, C, generator=g, device=dev).bfloat16()
    h = torch.randn(rows, C, generator=g, device=dev).bfloat16()
    w = (torch.randn(C, generator=g, device=dev) * 0.2 + (0.0 if mode == "plus_one" else 1.0)).bfloat16()
    gy = torch.randn(rows, C, generator=g, device=dev).bfloat16()
    gs = torch.randn(rows, C, generator=g, device=dev).bfloat16()
    eps = 1e-6
    xr = x.clone().requires_grad_(True)
    hr = h.clone().requires_grad_(True)
    x32 = x.float().cpu().requires_grad_(True)
    h32 = h.float().cpu().requires_grad_(True)
    if mode == "add":
        s, y = smelb.add_rmsnorm(hr, xr, w, eps, False)
        s32, y32 = O.add_rmsnorm(h32, x32, w.float().cpu(), eps, False)
        assert torch.equal(s.float().cpu(), s32.bfloat16().float())  # the residual sum rounds once, like torch
        (y.float() * gy.float()).sum().add_((s.float() * gs.float()).sum()).backward()
        (y32 * gy.float().cpu()).sum().add_((s32 * gs.float().cpu()).sum()).backward()
        close(xr.grad, x32.grad, "add_rmsnorm dx")
        close(hr.grad, h32.grad, "add_rmsnorm dh")
    else:
        ww = None if mode == "none" else w
        y = smelb.rmsnorm(xr, ww, eps, mode == "plus_one")
        y32 = O.rmsnorm(x32, None if ww is None else ww.float().cpu(), eps, mode == "plus_one")
        (y.float() * gy.float()).sum().backward()
        (y32 * gy.float().cpu()).sum().backward()
        close(xr.grad, x32.grad, f"rmsnorm {mode} dx")
    ref = y32.detach()
    diff = (y.float().cpu() - ref).abs()
    assert bool((diff <= ref.abs() * 2.0 ** -7 + 1e-6).all()), f"rmsnorm {mode}: max diff {diff.max().item():.3e}"
    assert smelb.read_status() == 0


def _gemma_inputs(d, dev):
    import smelb
    c = d["cfg"]
    bank = smelb.Int4Experts({"q": d["gu_q"].to(dev), "scale": d["gu_scale"].to(dev), "zero": d["gu_zero"].to(dev)},
                             {"q": d["dn_q"].to(dev), "scale": d["dn_scale"].to(dev), "zero": d["dn_zero"].to(dev)})
    sel = c["sel"]
    ex = smelb.LayerExperts(bank, sel, d["gu"][sel].bfloat16().to(dev), d["dn"][sel].bfloat16().to(dev),
                            act=c["act"])
    le = smelb.ExpertsLoRA(sel, c["H"], c["I"], c["r"], c["alpha"]).to(dev)
    ls = smelb.MLPLoRA(c["H"], c["S"], c["r"], c["alpha"]).to(dev)
    with torch.no_grad():
        for n in NAMES:
            getattr(le, n).copy_(d["lora_ex"][n])
            getattr(ls, n).copy_(d["lora_sh"][n])
    W = {k: v.bfloat16().to(dev) for k, v in d["W"].items()}
    return ex, smelb.LayerLoRA(le, ls), W


def test_route_gemma4_vs_oracle(dev, golden):
    """Routing indices equal the oracle's on the same bf16 input (ties: value desc, id asc); topv within 1e-2."""
    import smelb
    d = golden("gemma_block.pt")
    c = d["cfg"]
    _, _, W = _gemma_inputs(d, dev)
    h = d["h"].bfloat16().to(dev)
    probs, topv, topi = smelb.route_gemma4(h, W, c["K"], c["eps"])
    assert topv.dtype == torch.float32 and topi.dtype == torch.int64
    p32, v32, i32 = O.route_gemma4(h.cpu(), {k: v.cpu() for k, v in W.items()}, c["K"], c["eps"])
    agree = (topi.cpu() == i32).all(1).float().mean().item()
    assert agree >= 0.97, agree
    m = (topi.cpu() == i32).all(1)
    close(topv.cpu()[m], v32[m], "topv", rel=1e-2)
    close(probs.cpu(), p32, "probs", rel=2e-2)
    assert smelb.read_status() == 0


def test_gemma_block_vs_oracle_and_reference(dev, golden):
    """The Gemma 4 MoE block (smel/layer_runner.py:252-261): output, dh, dxm and all LoRA gradients against the fp64
    oracle with the GPU's routing forced, and the output against the reference's fp32 run where routing agrees."""
    import smelb
    d = golden("gemma_block.pt")
    c = d["cfg"]
    ex, lora, W = _gemma_inputs(d, dev)
    h = d["h"].bfloat16().to(dev).requires_grad_(True)
    xm = d["xm"].bfloat16().to(dev).requires_grad_(True)
    rec = {}
    out = smelb.moe_block_gemma4(h, xm, W, ex, c["K"], c["eps"], c["act"], lora,
                                 stats=lambda p, v, i: rec.update(p=p, v=v, i=i))
    gy = d["gy"].bfloat16().to(dev)
    out.backward(gy)
    topi = rec["i"].cpu()
    agree = (topi.sort(1).values == d["topi"].sort(1).values).all(1).float().mean().item()
    assert agree >= 0.9, agree
    dt = torch.float64
    s = c["alpha"] / c["r"]
    lex = {k: v.to(dt).requires_grad_(True) for k, v in d["lora_ex"].items()}
    lsh = {k: v.to(dt).requires_grad_(True) for k, v in d["lora_sh"].items()}
    h64 = h.detach().cpu().to(dt).requires_grad_(True)
    xm64 = xm.detach().cpu().to(dt).requires_grad_(True)
    W64 = {k: v.cpu().to(dt) for k, v in W.items()}
    gu = O.dequant_int4(d["gu_q"], d["gu_scale"], d["gu_zero"], dt)
    dn = O.dequant_int4(d["dn_q"], d["dn_scale"], d["dn_zero"], dt)
    sel = c["sel"]
    ref, _, ref_topv, _ = O.moe_block_gemma4(h64, xm64, W64, gu, dn, c["K"], c["eps"], sel,
                                             d["gu"][sel].bfloat16().to(dt), d["dn"][sel].bfloat16().to(dt),
                                             {**lex, "scale": s}, {**lsh, "scale": s}, c["act"], topi)
    ref.backward(gy.cpu().to(dt))
    close(out, ref, "out")
    close(rec["v"], ref_topv, "topv", rel=1e-2)
    close(h.grad, h64.grad, "dh")
    close(xm.grad, xm64.grad, "dxm")
    for n in NAMES:
        close(getattr(lora.experts, n).grad, lex[n].grad, "experts " + n)
        close(getattr(lora.shared, n).grad, lsh[n].grad, "dense " + n)
    m = (topi.sort(1).values == d["topi"].sort(1).values).all(1)
    close(out.float().cpu()[m], d["out"][m], "out vs reference", rel=3e-2, cos=0.999)
    assert smelb.read_status() == 0


class _LazyBank:
    """One expert of an int4 bank dequantized on the CPU on first access (the oracle's view of the frozen bank)."""

    def __init__(self, d, dtype):
        self.q, self.s, self.z = d["q"].cpu(), d["scale"].cpu(), d["zero"].cpu()
        self.shape = (self.q.shape[0], self.q.shape[1], self.q.shape[2] * 2)
        self.dtype, self.cache = dtype, {}

    def __getitem__(self, e):
        if e not in self.cache:
            self.cache[e] = O.dequant_int4(self.q[e], self.s[e], self.z[e]).to(self.dtype)
        return self.cache[e]


def test_gemma_config3_full_size(dev):
    """Config 3 at full size (H 2816, 128 experts top-8, I 704, dense GeGLU 2112 with LoRA, 4096 tokens, 116 int4 +
    12 LoRA experts, Zipf s=1.1): output, dh and dxm on every token and all 12 LoRA gradients against the oracle
    (fp32, the GPU's routing forced); routing against the oracle's own top-8 of the same bf16 inputs with every
    disagreeing row reported with its logit gap."""
    import smelb
    from smelb.synth import gemma_layer
    L = gemma_layer(device=dev, seed=0)
    meta, ex, lora, W = L["meta"], L["ex"], L["lora"], L["W"]
    assert abs(meta["share"] - 0.5) <= 0.02
    K, eps, sel = meta["K"], meta["eps"], meta["selected"]
    h = L["h"].clone().requires_grad_(True)
    xm = L["xm"].clone().requires_grad_(True)
    gy = torch.randn(h.shape, generator=torch.Generator(device=dev).manual_seed(9), device=dev).bfloat16()
    rec = {}
    out = smelb.moe_block_gemma4(h, xm, W, ex, K, eps, "gelu_tanh", lora,
                                 stats=lambda p, v, i: rec.update(p=p, v=v, i=i))
    out.backward(gy)
    assert smelb.read_status() == 0
    dt = torch.float32
    Wc = {k: v.cpu() for k, v in W.items()}
    # routing on the oracle's prologue (bf16 steps) with fp64 logits
    hc = h.detach().cpu()
    x = (hc.float() * torch.pow(hc.float().pow(2).mean(-1, keepdim=True) + eps, -0.5)).bfloat16()
    x = (x * Wc["router.scale"] * hc.shape[-1] ** -0.5).bfloat16()
    dis = O.routing_disagreements(rec["i"], x.double() @ Wc["router.proj.weight"].double().t(), K)
    print(f"routing: {len(dis)} of {hc.shape[0]} rows differ from the fp64 top-{K}; logit gaps "
          f"{[round(g, 5) for _, g in dis[:20]]}")
    # the Gemma router's logits are small (std ~0.02 around the Zipf bias), so bf16 rounding flips more near-ties
    # than at config 2; every flip must be a near-tie
    assert len(dis) <= 0.03 * hc.shape[0]
    assert all(g <= 2e-3 for _, g in dis), dis
    s = lora.experts.scale
    lex = {n: getattr(lora.experts, n).detach().cpu().to(dt).requires_grad_(True) for n in NAMES}
    lsh = {n: getattr(lora.shared, n).detach().cpu().to(dt).requires_grad_(True) for n in NAMES}
    h32 = hc.to(dt).requires_grad_(True)
    xm32 = xm.detach().cpu().to(dt).requires_grad_(True)
    W32 = {k: v.to(dt) for k, v in Wc.items()}
    ref, _, ref_topv, _ = O.moe_block_gemma4(h32, xm32, W32, _LazyBank(ex.frozen.gu, dt), _LazyBank(ex.frozen.dn, dt),
                                             K, eps, sel, ex.sel_gate_up.cpu().to(dt), ex.sel_down.cpu().to(dt),
                                             {**lex, "scale": s}, {**lsh, "scale": s}, "gelu_tanh", rec["i"].cpu())
    ref.backward(gy.cpu().to(dt))
    bad = []
    items = [("out", out, ref), ("topv", rec["v"], ref_topv), ("dh", h.grad, h32.grad), ("dxm", xm.grad, xm32.grad)]
    items += [("experts " + n, getattr(lora.experts, n).grad, lex[n].grad) for n in NAMES]
    items += [("dense " + n, getattr(lora.shared, n).grad, lsh[n].grad) for n in NAMES]
    for what, a, b in items:
        e, c = O.rel_err(a.float().cpu(), b.float()), O.cosine(a.float().cpu(), b.float())
        print(f"{what:>16s}: rel err {e:.3e} cosine {c:.7f}")
        if not (e <= 2e-2 and c >= 0.9999):
            bad.append(f"{what}: rel err {e:.3e}, cosine {c:.6f}")
    assert not bad, "; ".join(bad)
