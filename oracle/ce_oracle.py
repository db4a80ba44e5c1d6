"""CPU oracle for smelb's chunked cross-entropy — TEST INFRASTRUCTURE ONLY.

A restatement, on the CPU, of SMEL FT's chunked CE over a frozen LM head (smel/loss.py:12-156) and of the int8 row
format it reads (smel/quant.py:97-105). Only tests/ and bench.py's CPU baseline use it, as the checker / baseline;
the product (smel-ft_b200/smelb) never imports it.

Torch on the CPU in the dtype of the hidden rows, the reference's operation order: per vocabulary chunk a
matmul in that dtype, the logits taken to fp32 and capped, the running maximum / sum updated online, the softmax
numerators (times the cap's derivative) rounded to the hidden dtype before the second matmul.

Pinning: tests/golden/ce.pt holds the reference's own chunked_ce loss and gradient and its int8 rows
(tests/golden/make_golden.py --only ce); tests/test_ce.py checks this oracle against them.
"""
import torch


def quantize_int8_rows(w: torch.Tensor) -> dict:
    """smel/quant.py:97-101: symmetric per-row int8, s = max(amax|w| / 127, 1e-12) in fp32,
    q = clamp(round_half_even(w / s), -127, 127), the scale stored in bf16."""
    wf = w.float()
    s = (wf.abs().amax(-1, keepdim=True) / 127).clamp_min(1e-12)
    q = torch.round(wf / s).clamp_(-127, 127).to(torch.int8)
    return {"q": q, "scale": s.squeeze(-1).to(torch.bfloat16)}


def dequant_int8_rows(q: torch.Tensor, scale: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """smel/quant.py:104-105: q * scale in `dtype`."""
    return q.to(dtype) * scale.unsqueeze(-1).to(dtype)


def cap(z, softcap):
    """smel/loss.py:34-35."""
    return softcap * torch.tanh(z / softcap) if softcap else z


def _rows(w, q, v0, v1, dtype):
    """smel/loss.py:37-40."""
    if w is not None:
        return w[v0:v1].to(dtype)
    return dequant_int8_rows(q["q"][v0:v1], q["scale"][v0:v1], dtype)


def ce_chunk(h, tgt, w=None, q=None, vocab_chunk=32768, softcap=0.0, need_grad=True):
    """smel/loss.py:50-92 (_ce_chunk, the one-pass online gradient) for one token chunk. Returns the per-row losses
    (lse - target logit, fp32) and the fp32 gradient of their sum w.r.t. h (or None)."""
    n, H = h.shape
    V = w.shape[0] if w is not None else q["q"].shape[0]
    m = torch.full((n,), -float("inf"))
    s = torch.zeros(n)
    tgt_logit = torch.zeros(n)
    acc = torch.zeros(n, H) if need_grad else None
    tgt_row = torch.zeros(n, H) if need_grad else None
    tgt_d = torch.ones(n) if need_grad else None
    for v0 in range(0, V, vocab_chunk):
        v1 = min(V, v0 + vocab_chunk)
        W = _rows(w, q, v0, v1, h.dtype)
        lg = cap((h @ W.t()).float(), softcap)
        nm = torch.maximum(m, lg.amax(-1))
        r = (m - nm).exp()
        p = (lg - nm[:, None]).exp()
        s = s * r + p.sum(-1)
        idx = ((tgt >= v0) & (tgt < v1)).nonzero().squeeze(1)
        if idx.numel():
            col = tgt[idx] - v0
            tgt_logit[idx] = lg[idx, col]
            if need_grad:
                tgt_row[idx] = W[col].float()
                if softcap:
                    tgt_d[idx] = 1 - (lg[idx, col] / softcap) ** 2
        if need_grad:
            if softcap:
                p = p * (1 - (lg / softcap) ** 2)
            acc = acc * r[:, None] + (p.to(h.dtype) @ W).float()
        m = nm
    rows = m + s.log() - tgt_logit
    if not need_grad:
        return rows, None
    return rows, acc / s[:, None] - tgt_d[:, None] * tgt_row


def chunked_ce(h, tgt, denom, w=None, q=None, vocab_chunk=32768, token_chunk=1024, softcap=0.0, need_grad=True):
    """smel/loss.py:130-156: (loss, grad) with loss = sum of row losses / denom (fp32) and grad = (gradient / denom)
    in the dtype of h, over token chunks of `token_chunk` rows."""
    h, tgt = h.detach().cpu(), tgt.cpu()
    total = torch.zeros(())
    grads = []
    for t0 in range(0, h.shape[0], token_chunk):
        rows, g = ce_chunk(h[t0:t0 + token_chunk], tgt[t0:t0 + token_chunk], w, q, vocab_chunk, softcap, need_grad)
        total += rows.sum()
        if need_grad:
            grads.append(g)
    grad = (torch.cat(grads) / denom).to(h.dtype) if need_grad and grads else None
    return total / denom, grad


def cross_entropy_fp32(h, tgt, w_rows_fp32, softcap=0.0, denom=None):
    """Dense fp32 check of the same quantity (the reference tests' F.cross_entropy comparison,
    tests/test_data_loss.py:68-85, tests/test_gemma4.py:266-277): (loss, d loss / d h)."""
    hr = h.detach().float().cpu().requires_grad_(True)
    z = cap(hr @ w_rows_fp32.float().cpu().t(), softcap)
    loss = torch.nn.functional.cross_entropy(z, tgt.cpu(), reduction="sum") / (denom or h.shape[0])
    loss.backward()
    return loss.detach(), hr.grad
