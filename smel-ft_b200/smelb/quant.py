"""SMEL FT's group-wise asymmetric int4 format (smel/quant.py:1-94) and the int8 rows of the LM head
(smel/quant.py:97-105), on CUDA.

Format: w [..., K] -> q uint8 [..., K/2] (two nibbles per byte, the low nibble holds the even column),
scale / zero bf16 [..., K/group]; w ~= q * scale + zero. dequant_int4 computes q * scale + zero in fp32 and rounds
once to the output dtype (the reference's Triton kernel, smel/quant.py:51-67); dequant_int4_torch keeps the
reference's torch fallback rounding (smel/quant.py:87-94).
"""
import torch

from . import _lib

CLIP_SEARCH = (1.0, 0.95, 0.9, 0.85, 0.8)


def _codes(wg, lo, hi):
    """Step, base and codes of one clip candidate. Step and base are rounded to bf16 before use (they are stored
    that way), mirroring smel/quant.py:5-11."""
    step = ((hi - lo) / 15).clamp_min(1e-8).to(torch.bfloat16).float()
    base = lo.to(torch.bfloat16).float()
    codes = torch.round((wg - base) / step).clamp_(0, 15)
    return codes, step, base


def _quantize_slab(w, group, clip_search):
    K = w.shape[-1]
    wg = w.float().reshape(*w.shape[:-1], K // group, group)
    lo0, hi0 = wg.amin(-1, keepdim=True), wg.amax(-1, keepdim=True)
    center = (lo0 + hi0) / 2
    best_err = best_codes = best_step = best_base = None
    for c in clip_search or (1.0,):
        # candidate range shrunk towards the group center by c (same operation order as the reference)
        codes, step, base = _codes(wg, center + (lo0 - center) * c, center + (hi0 - center) * c)
        err = (codes * step + base - wg).pow(2).sum(-1, keepdim=True)
        if best_err is None:
            best_err, best_codes, best_step, best_base = err, codes, step, base
            continue
        take = err < best_err  # strictly better: the earlier candidate wins ties
        best_err = torch.where(take, err, best_err)
        best_codes = torch.where(take, codes, best_codes)
        best_step = torch.where(take, step, best_step)
        best_base = torch.where(take, base, best_base)
    codes = best_codes.to(torch.uint8).reshape(*w.shape[:-1], K)
    packed = codes[..., 0::2] | (codes[..., 1::2] << 4)
    return {"q": packed.contiguous(), "scale": best_step.squeeze(-1).to(torch.bfloat16),
            "zero": best_base.squeeze(-1).to(torch.bfloat16)}


def _quantize_kernel(w, clip_search):
    """Group-64 banks: one pass of `smelb_int4_quantize` (a warp per group, the candidates evaluated in
    registers)."""
    import ctypes
    K = w.shape[-1]
    w2 = w if w.dtype in (torch.bfloat16, torch.float32) else w.float()
    w2 = w2.contiguous()
    rows = w2.numel() // K
    lead = w.shape[:-1]
    q = torch.empty(*lead, K // 2, dtype=torch.uint8, device=w.device)
    scale = torch.empty(*lead, K // 64, dtype=torch.bfloat16, device=w.device)
    zero = torch.empty_like(scale)
    clip = (ctypes.c_float * len(clip_search))(*[float(c) for c in clip_search])
    _lib.call("smelb_int4_quantize", _lib.ptr(w2), 1 if w2.dtype == torch.float32 else 0, rows, K,
              ctypes.cast(clip, ctypes.c_void_p), len(clip_search), _lib.ptr(q), _lib.ptr(scale), _lib.ptr(zero),
              _lib.stream_ptr(w.device))
    return {"q": q, "scale": scale, "zero": zero}


def quantize_int4(w: torch.Tensor, group: int = 64, clip_search=CLIP_SEARCH) -> dict:
    """w [..., K] -> {q uint8 [..., K/2], scale bf16 [..., K/group], zero bf16 [..., K/group]}
    (smel/quant.py:14-44): per group the [min, max] range is shrunk by the clip factor with the smallest squared
    error. Group 64 (the fused kernels' format) runs the CUDA quantizer; other group sizes run the same steps as
    torch operations on the GPU, 16 experts at a time for 3-D banks to bound the fp32 temporaries."""
    if not w.is_cuda:
        raise _lib.SmelbError("quantize_int4: smelb quantizes on the GPU; move the weights to CUDA first")
    K = w.shape[-1]
    if K % group or group % 2:
        raise ValueError(f"quantize_int4: K={K} must be a multiple of an even group size (group={group})")
    clip_search = tuple(clip_search or (1.0,))
    if group == 64 and len(clip_search) <= 8:
        return _quantize_kernel(w, clip_search)
    if w.dim() == 3 and w.shape[0] > 16:
        parts = [_quantize_slab(w[i:i + 16], group, clip_search) for i in range(0, w.shape[0], 16)]
        return {k: torch.cat([p[k] for p in parts]) for k in parts[0]}
    return _quantize_slab(w, group, clip_search)


def _dequant(q, scale, zero, dtype, entry, what):
    if dtype not in (torch.bfloat16, torch.float32):
        raise _lib.SmelbError(f"{what}: output dtype {dtype} not supported (bf16 or fp32)")
    if q.dtype != torch.uint8 or scale.dtype != torch.bfloat16 or zero.dtype != torch.bfloat16:
        raise _lib.SmelbError(f"{what}: expects uint8 q and bf16 scale / zero")
    q, scale, zero = q.contiguous(), scale.contiguous(), zero.contiguous()
    half_k, groups = q.shape[-1], scale.shape[-1]
    out = torch.empty(*q.shape[:-1], half_k * 2, device=q.device, dtype=dtype)
    rows = q.numel() // max(half_k, 1)
    _lib.call(entry, _lib.ptr(q), _lib.ptr(scale), _lib.ptr(zero), _lib.ptr(out), rows, half_k * 2, groups,
              1 if dtype == torch.float32 else 0, _lib.stream_ptr(q.device))
    return out


def dequant_int4(q: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """q [..., K/2], scale/zero [..., G] -> [..., K] in `dtype` (bf16 or fp32), on the GPU: q * scale + zero in fp32,
    rounded once to `dtype` (the reference's Triton kernel, smel/quant.py:51-67, 74-84)."""
    return _dequant(q, scale, zero, dtype, "smelb_int4_dequant", "dequant_int4")


def dequant_int4_torch(q, scale, zero, dtype=torch.bfloat16):
    """smel/quant.py:87-94: the same dequant with torch's operation-by-operation rounding in `dtype`: for bf16 the
    product q * scale is rounded to bf16 before zero is added and the sum is rounded again (it differs from
    dequant_int4 on many weights, exactly as in the reference). fp32 output equals dequant_int4."""
    return _dequant(q, scale, zero, dtype, "smelb_int4_dequant_stepwise", "dequant_int4_torch")


def pack_sz(scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    """(scale | zero << 16) pairs transposed to [nw, groups, rows] uint32 (stored as int32): the layout the fused
    expert GEMMs stage per k-block. scale / zero bf16 [nw, rows, groups]."""
    scale, zero = scale.contiguous(), zero.contiguous()
    nw, rows, groups = scale.shape
    out = torch.empty(nw, groups, rows, device=scale.device, dtype=torch.int32)
    _lib.call("smelb_int4_pack_sz", _lib.ptr(scale), _lib.ptr(zero), _lib.ptr(out), nw, rows, groups,
              _lib.stream_ptr(scale.device))
    return out


def quantize_int8_rows(w: torch.Tensor) -> dict:
    """Symmetric per-row int8 for the LM head (smel/quant.py:97-101), on the GPU: w [..., H] (bf16 or fp32) ->
    {q int8 [..., H], scale bf16 [...]}, s = max(amax|w| / 127, 1e-12), q = clamp(round(w / s), -127, 127)."""
    if not w.is_cuda:
        raise _lib.SmelbError("quantize_int8_rows: smelb quantizes on the GPU; move the weights to CUDA first")
    w2 = w if w.dtype in (torch.bfloat16, torch.float32) else w.float()
    w2 = w2.contiguous()
    H = w2.shape[-1]
    rows = w2.numel() // max(H, 1)
    q = torch.empty(w2.shape, dtype=torch.int8, device=w.device)
    scale = torch.empty(w2.shape[:-1], dtype=torch.bfloat16, device=w.device)
    _lib.call("smelb_int8_rows_quantize", _lib.ptr(w2), 1 if w2.dtype == torch.float32 else 0, rows, H, _lib.ptr(q),
              _lib.ptr(scale), _lib.stream_ptr(w.device))
    return {"q": q, "scale": scale}


def dequant_int8_rows(q: torch.Tensor, scale: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """q * scale in `dtype` (bf16 or fp32) on the GPU (smel/quant.py:104-105)."""
    if dtype not in (torch.bfloat16, torch.float32):
        raise _lib.SmelbError(f"dequant_int8_rows: output dtype {dtype} not supported (bf16 or fp32)")
    if q.dtype != torch.int8 or scale.dtype != torch.bfloat16:
        raise _lib.SmelbError("dequant_int8_rows: expects int8 q and a bf16 scale")
    q, scale = q.contiguous(), scale.contiguous()
    H = q.shape[-1]
    out = torch.empty(q.shape, dtype=dtype, device=q.device)
    _lib.call("smelb_int8_rows_dequant", _lib.ptr(q), _lib.ptr(scale), q.numel() // max(H, 1), H, _lib.ptr(out),
              1 if dtype == torch.float32 else 0, _lib.stream_ptr(q.device))
    return out


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in fp32 (smel/quant.py:108-110)."""
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
