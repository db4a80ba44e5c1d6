"""The layer-major driver (smelb/runner.py) on a stack of three synthetic MoE layers with LoRA on the GPU, two
micro-batches: forward without autograd, recompute + backward in reverse layer order. Against one autograd pass per
micro-batch through the same stack the inputs' gradients and every layer's LoRA gradients are bit-identical (the same
kernels on the same inputs, deterministic reductions); the top layer's LoRA gradients match the fp64 oracle on that
layer's checkpointed input and the upstream gradient (max relative error 2e-2, cosine 0.9999)."""
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")


def test_layer_major_stack_matches_autograd_and_oracle():
    import smelb
    from smelb.runner import LayerMajorRunner
    from smelb.synth import qwen_layer
    dev = torch.device("cuda:0")
    K, nL = 4, 3
    layers, loras = {}, {}
    for l in range(nL):
        Ly = qwen_layer(T=300, H=256, E=16, K=K, I=128, S=128, n_sel=3, r=8, alpha=16.0, seed=40 + l, device=dev)
        layers[l] = (Ly["W"], Ly["ex"])
        loras[l] = Ly["lora"]
        if l == 0:
            x0 = Ly["x"]
    block = smelb.BlockLoRA(loras)
    xs = [x0[:170].contiguous(), x0[170:].contiguous()]
    g = torch.Generator(device=dev).manual_seed(7)
    gys = [torch.randn(x.shape, generator=g, device=dev).bfloat16() for x in xs]
    params = list(block.parameters())
    # reference: autograd through the stack
    ref_dx = []
    for x, gy in zip(xs, gys):
        xr = x.clone().requires_grad_(True)
        h = xr
        for l in range(nL):
            h = h + smelb.moe_forward(h, layers[l][0], layers[l][1], K, loras[l])
        h.backward(gy)
        ref_dx.append(xr.grad)
    ref_g = [p.grad.clone() for p in params]
    for p in params:
        p.grad = None
    runner = LayerMajorRunner(layers, range(nL), lora=block, top_k=K)
    routes = {}
    hs, ckpt = runner.forward([x.clone() for x in xs], keep_ckpt=True,
                              stats_cb=lambda l, m, p, v, t: routes.update({(l, m): t.clone()}))
    top_in = [c.clone() for c in ckpt[nL - 1]]
    dx = runner.backward(ckpt, [gy.clone() for gy in gys])
    for a, b in zip(dx, ref_dx):
        assert torch.equal(a, b)
    for p, r in zip(params, ref_g):
        assert torch.equal(p.grad, r)
    # the top layer against the oracle from its checkpointed inputs
    W, ex = layers[nL - 1]
    lo = loras[nL - 1]
    dt = torch.float64
    lex = {n: getattr(lo.experts, n).detach().cpu().to(dt).requires_grad_(True) for n in NAMES}
    lsh = {n: getattr(lo.shared, n).detach().cpu().to(dt).requires_grad_(True) for n in NAMES}
    gu = torch.stack([O.dequant_int4(ex.frozen.gu["q"][e].cpu(), ex.frozen.gu["scale"][e].cpu(),
                                     ex.frozen.gu["zero"][e].cpu()) for e in range(ex.E)]).to(dt)
    dn = torch.stack([O.dequant_int4(ex.frozen.dn["q"][e].cpu(), ex.frozen.dn["scale"][e].cpu(),
                                     ex.frozen.dn["zero"][e].cpu()) for e in range(ex.E)]).to(dt)
    s = lo.experts.scale
    for m in range(len(xs)):
        h64 = top_in[m].cpu().to(dt)
        out, _, _, _ = O.moe_layer(h64, {k: v.cpu().to(dt) for k, v in W.items()}, gu, dn, K,
                                   ex.sel_ids.tolist(), ex.sel_gate_up.cpu().to(dt), ex.sel_down.cpu().to(dt),
                                   {**lex, "scale": s}, {**lsh, "scale": s}, topi=routes[(nL - 1, m)].cpu())
        out.backward(gys[m].cpu().to(dt))
    for n in NAMES:
        for what, got, want in ((f"experts {n}", getattr(lo.experts, n).grad, lex[n].grad),
                                (f"shared {n}", getattr(lo.shared, n).grad, lsh[n].grad)):
            e, c = O.rel_err(got.float().cpu(), want), O.cosine(got.float().cpu(), want)
            assert e <= 2e-2 and c >= 0.9999, f"{what}: rel err {e:.3e} cosine {c:.6f}"
    assert smelb.read_status() == 0
