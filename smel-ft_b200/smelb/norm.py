"""Row norms around the MoE layer (smel/norm.py; torch form smel/layer_runner.py:110-130) on the smelb kernels.

    rmsnorm(x, w, eps, plus_one)       y = x * rstd * (1 + w) (Qwen3.5/3.6), x * rstd * w (Gemma 4), x * rstd (w None)
    add_rmsnorm(h, x, w, eps, plus_one) (s, y): s = h + x (the residual add, rounded like torch's), y = rmsnorm(s)
    router_prologue_gemma4(h, scale, eps)  the Gemma 4 router input of smel/moe.py:170-176:
                                        bf16(bf16(bf16(h * rstd) * scale) * H^-0.5)

fp32 math with one rounding to the activation dtype, as the reference; the norm weights are frozen (SMEL trains
LoRA only), so the backward returns input gradients only. One warp per row, bf16 rows with C % 8 == 0.
"""
import torch

from . import _lib


def _bf16_rows(t, what):
    if not t.is_cuda:
        raise _lib.SmelbError(f"{what}: smelb runs on CUDA tensors only")
    if t.dtype != torch.bfloat16:
        raise _lib.SmelbError(f"{what}: expected bf16, got {t.dtype}")
    return t.reshape(-1, t.shape[-1]).contiguous()


def _w(w, C, what):
    if w is None:
        return None
    if w.shape != (C,):
        raise _lib.SmelbError(f"{what}: weight of shape {tuple(w.shape)} for {C} columns")
    return w.detach().to(torch.bfloat16).contiguous()


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, w_mode, post_scale, post_mul):
        x2 = _bf16_rows(x, "rmsnorm: x")
        rows, C = x2.shape
        y = torch.empty_like(x2)
        rstd = torch.empty(rows, dtype=torch.float32, device=x2.device)
        _lib.call("smelb_rmsnorm_fwd", _lib.ptr(x2), None, _lib.ptr(w), w_mode, _lib.ptr(post_scale), post_mul,
                  float(eps), rows, C, None, _lib.ptr(y), _lib.ptr(rstd), _lib.stream_ptr(x2.device))
        ctx.save_for_backward(x2, rstd)
        ctx.w, ctx.w_mode, ctx.post_scale, ctx.post_mul, ctx.shape = w, w_mode, post_scale, post_mul, x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, rstd = ctx.saved_tensors
        rows, C = x2.shape
        dy = dy.to(torch.bfloat16).reshape(rows, C).contiguous()
        dx = torch.empty_like(x2)
        _lib.call("smelb_rmsnorm_bwd", _lib.ptr(dy), _lib.ptr(x2), _lib.ptr(ctx.w), ctx.w_mode,
                  _lib.ptr(ctx.post_scale), ctx.post_mul, _lib.ptr(rstd), None, rows, C, _lib.ptr(dx),
                  _lib.stream_ptr(x2.device))
        return dx.view(ctx.shape), None, None, None, None, None


class _AddRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, x, w, eps, w_mode):
        h2, x2 = _bf16_rows(h, "add_rmsnorm: h"), _bf16_rows(x, "add_rmsnorm: x")
        if h2.shape != x2.shape:
            raise _lib.SmelbError(f"add_rmsnorm: shapes {tuple(h.shape)} and {tuple(x.shape)}")
        rows, C = h2.shape
        s, y = torch.empty_like(h2), torch.empty_like(h2)
        rstd = torch.empty(rows, dtype=torch.float32, device=h2.device)
        _lib.call("smelb_rmsnorm_fwd", _lib.ptr(x2), _lib.ptr(h2), _lib.ptr(w), w_mode, None, 0.0, float(eps), rows, C,
                  _lib.ptr(s), _lib.ptr(y), _lib.ptr(rstd), _lib.stream_ptr(h2.device))
        ctx.save_for_backward(s, rstd)
        ctx.w, ctx.w_mode, ctx.shape = w, w_mode, h.shape
        ctx.set_materialize_grads(False)
        return s.view(h.shape), y.view(h.shape)

    @staticmethod
    def backward(ctx, ds, dy):
        s, rstd = ctx.saved_tensors
        rows, C = s.shape
        if dy is None:  # only the sum was used
            d = ds.to(torch.bfloat16).reshape(rows, C)
            return d.view(ctx.shape), d.view(ctx.shape), None, None, None
        dy = dy.to(torch.bfloat16).reshape(rows, C).contiguous()
        ds2 = ds.to(torch.bfloat16).reshape(rows, C).contiguous() if ds is not None else None
        d = torch.empty_like(s)
        _lib.call("smelb_rmsnorm_bwd", _lib.ptr(dy), _lib.ptr(s), _lib.ptr(ctx.w), ctx.w_mode, None, 0.0,
                  _lib.ptr(rstd), _lib.ptr(ds2), rows, C, _lib.ptr(d), _lib.stream_ptr(s.device))
        return d.view(ctx.shape), d.view(ctx.shape), None, None, None


def rmsnorm(x, w, eps, plus_one=True):
    """smel/layer_runner.py:110-121 (smel/norm.py rmsnorm): x * rstd * (1 + w), x * rstd * w (plus_one False) or
    x * rstd (w None), fp32 math, one rounding; differentiable in x."""
    C = x.shape[-1]
    mode = 0 if w is None else (2 if plus_one else 1)
    return _RMSNormFn.apply(x, _w(w, C, "rmsnorm"), eps, mode, None, 0.0)


def add_rmsnorm(h, x, w, eps, plus_one=True):
    """smel/layer_runner.py:124-130: (h + x, rmsnorm(h + x, w)) in one kernel each way."""
    return _AddRMSNormFn.apply(h, x, _w(w, h.shape[-1], "add_rmsnorm"), eps, 2 if plus_one else 1)


def router_prologue_gemma4(h, scale, eps):
    """The Gemma 4 router input (smel/moe.py:173-175): the weightless RMSNorm of h rounded to h's dtype, times
    router.scale (rounded), times H^-0.5 (rounded); differentiable in h."""
    C = h.shape[-1]
    return _RMSNormFn.apply(h, None, eps, 0, _w(scale, C, "router.scale"), float(C ** -0.5))
