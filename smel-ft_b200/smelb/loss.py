"""Chunked cross-entropy over a frozen LM head (smel/loss.py:1-156), on CUDA.

Same interface as the reference: LMHead (bf16 rows or int8 rows, vocab_chunk, optional final-logit softcap) and
chunked_ce(h, head, tgt, denom, token_chunk, need_grad), whose backward returns the gradient computed in the forward
pass (the head is frozen). The [N, V] logits are never materialised.

B200 design (libsmelb.so, smelb_chunked_ce): one pass over the vocabulary chunks, each applied to every token chunk
in turn (the online state of all rows is kept, so an int8 head is dequantised once per call); per chunk the logits
come from the MoE layer's tcgen05 GEMM engine (head rows as the MMA's M side, tokens as N) in bf16, a row
kernel does the online max / sum, takes the target's logit and head row, and overwrites the logits in place with the
softmax numerators times the cap's derivative (bf16, as the reference's p.to(h.dtype)); a second GEMM multiplies them
by the same head rows (MN-major, split along the chunk into fp32 partials that fill the SMs) and a last kernel
rescales the fp32 gradient accumulator. An int8 head's chunk is dequantised into a bf16 buffer of the workspace.
Only the hidden dtype bf16 is supported (the reference's training dtype).
"""
import torch

from . import _lib
from .quant import dequant_int8_rows, quantize_int8_rows


class LMHead:
    """smel/loss.py:12-47."""

    def __init__(self, weight: torch.Tensor | None = None, int8: dict | None = None, vocab_chunk: int = 32768,
                 softcap: float = 0.0):
        assert (weight is None) != (int8 is None)
        self.w, self.q = weight, int8
        self.vocab = weight.shape[0] if weight is not None else int8["q"].shape[0]
        self.vocab_chunk = vocab_chunk
        self.softcap = float(softcap or 0.0)

    @classmethod
    def from_weight(cls, w, int8=False, vocab_chunk=32768, softcap=0.0):
        if int8:
            return cls(int8=quantize_int8_rows(w), vocab_chunk=vocab_chunk, softcap=softcap)
        return cls(weight=w, vocab_chunk=vocab_chunk, softcap=softcap)

    def to(self, device):
        if self.w is not None:
            return LMHead(weight=self.w.to(device), vocab_chunk=self.vocab_chunk, softcap=self.softcap)
        return LMHead(int8={k: v.to(device) for k, v in self.q.items()}, vocab_chunk=self.vocab_chunk,
                      softcap=self.softcap)

    def cap(self, z: torch.Tensor) -> torch.Tensor:
        return self.softcap * torch.tanh(z / self.softcap) if self.softcap else z

    def rows(self, v0, v1, dtype):
        if self.w is not None:
            return self.w[v0:v1].to(dtype)
        return dequant_int8_rows(self.q["q"][v0:v1], self.q["scale"][v0:v1], dtype)

    def chunks(self):
        for v0 in range(0, self.vocab, self.vocab_chunk):
            yield v0, min(self.vocab, v0 + self.vocab_chunk)

    def logits(self, h):
        """cap(h @ W^T) in fp32 [N, V] (smel/loss.py:45-47), chunk by chunk on the GEMM engine."""
        h = _check_h(h, "LMHead.logits")
        N, H = h.shape
        keep, (wp, qp, sp), int8 = _head_ptrs(self, h.device)
        out = torch.empty(N, self.vocab, dtype=torch.float32, device=h.device)
        if N == 0:
            return out
        vc = min(self.vocab_chunk, self.vocab)
        nb = int(_lib.load().smelb_lm_logits_workspace_bytes(N, H, vc, 1 if int8 else 0))
        ws = torch.empty(nb, dtype=torch.uint8, device=h.device)
        _lib.call("smelb_lm_logits", _lib.ptr(h), N, H, wp, qp, sp, self.vocab, self.vocab_chunk, self.softcap,
                  _lib.ptr(out), _lib.ptr(ws), nb, _lib.stream_ptr(h.device))
        return out


def _head_ptrs(head, device):
    """(tensors to keep alive, (w, q, scale) pointers, int8?) of a head: this module's LMHead or the reference's
    (smel/loss.py:12-47), which has the same fields (w or q, vocab, vocab_chunk, softcap)."""
    if head.w is not None:
        w = head.w if head.w.dtype == torch.bfloat16 else head.w.to(torch.bfloat16)
        w = w.contiguous()
        if w.device != device:
            raise _lib.SmelbError(f"LMHead: head on {w.device}, hidden rows on {device}")
        return (w,), (_lib.ptr(w), None, None), False
    q, s = head.q["q"].contiguous(), head.q["scale"].contiguous()
    if q.device != device:
        raise _lib.SmelbError(f"LMHead: head on {q.device}, hidden rows on {device}")
    return (q, s), (None, _lib.ptr(q), _lib.ptr(s)), True


def _check_h(h, who):
    if not h.is_cuda:
        raise _lib.SmelbError(f"{who}: smelb runs on CUDA tensors only")
    if h.dtype != torch.bfloat16:
        raise _lib.SmelbError(f"{who}: hidden rows must be bf16 (got {h.dtype})")
    if h.dim() != 2 or h.shape[1] % 64:
        raise _lib.SmelbError(f"{who}: h must be [N, H] with H a multiple of 64 (got {tuple(h.shape)})")
    return h.contiguous()


def _run(h, head: LMHead, tgt, denom, token_chunk, need_grad):
    """One smelb_chunked_ce call: (loss fp32 0-dim, per-row losses fp32 [N], gradient bf16 [N, H] or None)."""
    N, H = h.shape
    keep, (wp, qp, sp), int8 = _head_ptrs(head, h.device)
    tgt = tgt.to(device=h.device, dtype=torch.int64).contiguous()
    tc = max(1, min(int(token_chunk), N))
    vc = min(head.vocab_chunk, head.vocab)
    nb = int(_lib.load().smelb_chunked_ce_workspace_bytes(N, tc, H, vc, 1 if int8 else 0, 1 if need_grad else 0))
    ws = torch.empty(nb, dtype=torch.uint8, device=h.device)
    rows = torch.empty(N, dtype=torch.float32, device=h.device)
    loss = torch.empty((), dtype=torch.float32, device=h.device)
    gh = torch.empty(N, H, dtype=torch.bfloat16, device=h.device) if need_grad else None
    _lib.call("smelb_chunked_ce", _lib.ptr(h), _lib.ptr(tgt), N, H, wp, qp, sp, head.vocab, head.vocab_chunk,
              int(token_chunk), head.softcap, float(denom), _lib.ptr(rows), _lib.ptr(loss), _lib.ptr(gh), _lib.ptr(ws),
              nb, _lib.stream_ptr(h.device))
    return loss, rows, gh


class _ChunkedCE(torch.autograd.Function):
    """smel/loss.py:130-146."""

    @staticmethod
    def forward(ctx, h, head, tgt, denom, token_chunk, need_grad):
        loss, _, gh = _run(_check_h(h, "chunked_ce"), head, tgt, denom, token_chunk, need_grad)
        if need_grad:
            ctx.grad = gh
        return loss

    @staticmethod
    def backward(ctx, go):
        return ctx.grad * go.to(ctx.grad.dtype), None, None, None, None, None


def chunked_ce(h, head: LMHead, tgt, denom: float, token_chunk: int = 1024, need_grad: bool = True):
    """sum_t CE(h_t @ W.T, tgt_t) / denom (smel/loss.py:149-156). h: [N, H] bf16 (final-normed, only supervised
    rows), tgt: [N] long."""
    if h.shape[0] == 0:
        return (h.float().sum() * 0.0)
    if need_grad and h.requires_grad:
        return _ChunkedCE.apply(h, head, tgt, float(denom), token_chunk, True)
    with torch.no_grad():
        return _ChunkedCE.apply(h, head, tgt, float(denom), token_chunk, False)


def chunked_ce_rows(h, head: LMHead, tgt, token_chunk: int = 1024):
    """Per-row losses lse - target logit (fp32 [N]), without the gradient."""
    h = _check_h(h, "chunked_ce_rows")
    if h.shape[0] == 0:
        return torch.zeros(0, dtype=torch.float32, device=h.device)
    return _run(h, head, tgt, 1.0, token_chunk, False)[1]
