"""The layer-major driver (smelb/runner.py, smel/layer_runner.py:295-371) on the CPU with a plain torch layer
function: forward over all micro-batches layer by layer without autograd, then recompute + backward in reverse layer
order, against one autograd pass through the same stack per micro-batch (inputs' gradients and the parameters'
accumulated gradients equal to fp64 rounding)."""
import torch


def _layers(n, H, gen):
    return [(torch.randn(H, H, generator=gen, dtype=torch.float64) * 0.3).requires_grad_(True) for _ in range(n)]


def _fn(h, layer, lora, stats=None):
    if stats is not None:
        stats(None, None, None)
    return h + torch.tanh(h @ layer)


def test_layer_major_matches_stacked_autograd():
    from smelb.runner import LayerMajorRunner
    g = torch.Generator().manual_seed(0)
    H, L, M = 16, 4, 3
    Ws = _layers(L, H, g)
    xs = [torch.randn(5 + m, H, generator=g, dtype=torch.float64) for m in range(M)]
    gys = [torch.randn(5 + m, H, generator=g, dtype=torch.float64) for m in range(M)]
    # reference: autograd through the whole stack, micro-batch by micro-batch
    ref_dx = []
    for x, gy in zip(xs, gys):
        xr = x.clone().requires_grad_(True)
        h = xr
        for W in Ws:
            h = _fn(h, W, None)
        h.backward(gy)
        ref_dx.append(xr.grad)
    ref_dW = [W.grad.clone() for W in Ws]
    for W in Ws:
        W.grad = None
    calls = []
    runner = LayerMajorRunner({l: W for l, W in enumerate(Ws)}, range(L), layer_fn=_fn)
    hs, ckpt = runner.forward([x.clone() for x in xs], keep_ckpt=True,
                              stats_cb=lambda l, m, p, v, t: calls.append((l, m)))
    assert calls == [(l, m) for l in range(L) for m in range(M)]  # layer-major order
    assert all(not h.requires_grad for h in hs)
    dx = runner.backward(ckpt, [gy.clone() for gy in gys])
    assert all(v is None for c in ckpt.values() for v in c)  # checkpoints are released as the backward passes
    for a, b in zip(dx, ref_dx):
        assert torch.allclose(a, b, rtol=1e-12, atol=1e-12)
    for W, r in zip(Ws, ref_dW):
        assert torch.allclose(W.grad, r, rtol=1e-12, atol=1e-12)
    # train_step: the head's gradients come from grad_fn
    for W in Ws:
        W.grad = None
    dx2, extra = runner.train_step([x.clone() for x in xs], lambda top: ([gy.clone() for gy in gys], len(top)))
    assert extra == M and all(torch.allclose(a, b) for a, b in zip(dx2, ref_dx))
