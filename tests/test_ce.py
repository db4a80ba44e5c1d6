"""Chunked cross-entropy over a frozen LM head (smelb/loss.py, smel/loss.py:12-156) and the int8 rows it reads
(smel/quant.py:97-105).

CPU: the oracle (oracle/ce_oracle.py) against the reference's own outputs (tests/golden/ce.pt, written by
tests/golden/make_golden.py --only ce), and the API's refusal of CPU tensors.
GPU: smelb_chunked_ce against the same fixtures (the reference's bf16 loss and gradient; the kernels accumulate the
GEMMs in fp32 in another order, so the bar is a tolerance: loss within 2e-3 relative, gradient rel err < 1e-2 and
cosine > 0.9999), against a dense fp32 cross-entropy (the reference tests' bar: |loss| 1e-2, gradient 2e-2), the
int8 quantizer bit-exact, the loss-only path, invariance of the per-row losses to the token chunk, and a larger
head against a dense fp32 computation on the GPU."""
import pytest
import torch

from oracle import ce_oracle as O

CASES = ("bf16", "int8", "softcap")


def _q(c):
    return {"q": c["q"], "scale": c["scale"]} if "q" in c else None


def _cos(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-30))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_chunked_ce(golden, name):
    c = golden("ce.pt")[name]
    loss, grad = O.chunked_ce(c["h"], c["tgt"], c["denom"], c.get("w"), _q(c), c["vocab_chunk"], c["token_chunk"],
                              c["softcap"])
    assert torch.equal(loss, c["loss"])
    assert torch.equal(grad, c["grad"])
    if "loss_nograd" in c:
        l2, g2 = O.chunked_ce(c["h"], c["tgt"], c["denom"], c.get("w"), _q(c), c["vocab_chunk"], c["token_chunk"],
                              c["softcap"], need_grad=False)
        assert g2 is None and torch.equal(l2, c["loss_nograd"])


def test_oracle_int8_rows_match_reference(golden):
    d = golden("ce.pt")
    q = O.quantize_int8_rows(d["bf16"]["w"])
    assert torch.equal(q["q"], d["int8"]["q"]) and torch.equal(q["scale"].view(torch.int16),
                                                                d["int8"]["scale"].view(torch.int16))


def test_head_fields_are_read_duck_typed():
    """chunked_ce reads only the head's fields (w or q, vocab, vocab_chunk, softcap), so a head built by the
    reference's LMHead (same fields) reaches the same device check instead of failing on a missing method."""
    import types
    import smelb
    head = types.SimpleNamespace(w=torch.randn(100, 64).bfloat16(), q=None, vocab=100, vocab_chunk=64, softcap=0.0)
    from smelb import loss as L
    with pytest.raises(smelb.SmelbError, match="head on cpu"):
        L._head_ptrs(head, torch.device("cuda", 0))


def test_cpu_tensors_are_rejected():
    import smelb
    w = torch.randn(100, 64).bfloat16()
    with pytest.raises(smelb.SmelbError):
        smelb.quantize_int8_rows(w)
    head = smelb.LMHead.from_weight(w, vocab_chunk=64)
    with pytest.raises(smelb.SmelbError):
        smelb.chunked_ce(torch.randn(4, 64).bfloat16().requires_grad_(True), head, torch.zeros(4, dtype=torch.long),
                         4.0)


# ------------------------------------------------------------------------------------------------------ GPU
def _head(c, dev, vocab_chunk=None):
    import smelb
    vc = vocab_chunk or c["vocab_chunk"]
    if "q" in c:
        return smelb.LMHead(int8={"q": c["q"].to(dev), "scale": c["scale"].to(dev)}, vocab_chunk=vc,
                            softcap=c["softcap"])
    return smelb.LMHead(weight=c["w"].to(dev), vocab_chunk=vc, softcap=c["softcap"])


def _run(c, dev, token_chunk=None, vocab_chunk=None):
    import smelb
    h = c["h"].to(dev).requires_grad_(True)
    loss = smelb.chunked_ce(h, _head(c, dev, vocab_chunk), c["tgt"].to(dev), c["denom"],
                            token_chunk or c["token_chunk"])
    loss.backward()
    return loss.detach().cpu(), h.grad.cpu()


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_chunked_ce_matches_reference(golden, name):
    c = golden("ce.pt")[name]
    dev = torch.device("cuda", 0)
    loss, grad = _run(c, dev)
    assert grad.dtype == torch.bfloat16 and grad.shape == c["h"].shape
    assert abs(float(loss) - float(c["loss"])) <= 2e-3 * abs(float(c["loss"])), (float(loss), float(c["loss"]))
    rel = float((grad.float() - c["grad"].float()).norm() / c["grad"].float().norm())
    assert rel < 1e-2 and _cos(grad, c["grad"]) > 0.9999, (rel, _cos(grad, c["grad"]))
    # the reference tests' own bar against a dense fp32 cross-entropy
    w = c["w"] if "w" in c else O.dequant_int8_rows(c["q"], c["scale"], torch.float32)
    lr, gr = O.cross_entropy_fp32(c["h"], c["tgt"], w, c["softcap"], c["denom"])
    assert abs(float(loss) - float(lr)) < 1e-2
    assert float((grad.float() - gr).norm() / gr.norm()) < 2e-2


@pytest.mark.gpu
def test_chunked_ce_loss_only_and_backward_scale(golden):
    import smelb
    c = golden("ce.pt")["softcap"]
    dev = torch.device("cuda", 0)
    head = _head(c, dev)
    with torch.no_grad():
        l0 = smelb.chunked_ce(c["h"].to(dev), head, c["tgt"].to(dev), c["denom"], c["token_chunk"])
    l1, g1 = _run(c, dev)
    assert torch.equal(l0.cpu(), l1)  # the loss does not depend on whether the gradient is formed
    assert abs(float(l0) - float(c["loss_nograd"])) <= 2e-3 * abs(float(c["loss_nograd"]))
    h = c["h"].to(dev).requires_grad_(True)
    (3.0 * smelb.chunked_ce(h, head, c["tgt"].to(dev), c["denom"], c["token_chunk"])).backward()
    assert torch.equal(h.grad.cpu(), (g1 * torch.tensor(3.0, dtype=torch.bfloat16)))


@pytest.mark.gpu
def test_per_row_losses_do_not_depend_on_token_chunk(golden):
    from smelb import loss as L
    c = golden("ce.pt")["bf16"]
    dev = torch.device("cuda", 0)
    head = _head(c, dev)
    h, t = c["h"].to(dev), c["tgt"].to(dev)
    ref = L.chunked_ce_rows(h, head, t, token_chunk=1024)
    for tc in (1, 7, 64, 193):
        assert torch.equal(L.chunked_ce_rows(h, head, t, token_chunk=tc), ref), tc
    lo, _ = O.ce_chunk(c["h"], c["tgt"], w=c["w"], vocab_chunk=c["vocab_chunk"], need_grad=False)
    assert float((ref.cpu() - lo).abs().max()) < 2e-2


@pytest.mark.gpu
def test_int8_rows_quantizer_bit_exact(golden):
    import smelb
    d = golden("ce.pt")
    dev = torch.device("cuda", 0)
    q = smelb.quantize_int8_rows(d["bf16"]["w"].to(dev))
    assert torch.equal(q["q"].cpu(), d["int8"]["q"])
    assert torch.equal(q["scale"].cpu().view(torch.int16), d["int8"]["scale"].view(torch.int16))
    wf = torch.randn(37, 200, generator=torch.Generator().manual_seed(3)) * 0.1
    wf[5] = 0.0  # an all-zero row: the scale's 1e-12 floor
    qf, of = smelb.quantize_int8_rows(wf.to(dev)), O.quantize_int8_rows(wf)
    assert torch.equal(qf["q"].cpu(), of["q"]) and torch.equal(qf["scale"].cpu().view(torch.int16),
                                                               of["scale"].view(torch.int16))
    for dt in (torch.bfloat16, torch.float32):
        out = smelb.dequant_int8_rows(qf["q"], qf["scale"], dt).cpu()
        assert torch.equal(out, O.dequant_int8_rows(of["q"], of["scale"], dt))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ("bf16", "softcap"))
def test_lm_head_logits(golden, name):
    c = golden("ce.pt")[name]
    dev = torch.device("cuda", 0)
    z = _head(c, dev).logits(c["h"].to(dev)).cpu()
    ref = O.cap((c["h"] @ c["w"].t()).float(), c["softcap"])
    assert z.shape == ref.shape and z.dtype == torch.float32
    assert float((z - ref).norm() / ref.norm()) < 5e-3


@pytest.mark.gpu
def test_empty_rows():
    import smelb
    dev = torch.device("cuda", 0)
    head = smelb.LMHead.from_weight(torch.randn(300, 64, device=dev).bfloat16(), vocab_chunk=128)
    h = torch.zeros(0, 64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    loss = smelb.chunked_ce(h, head, torch.zeros(0, dtype=torch.long, device=dev), 1.0)
    loss.backward()
    assert float(loss) == 0.0 and h.grad.shape == (0, 64)


@pytest.mark.gpu
@pytest.mark.parametrize("int8", (False, True))
def test_large_head_against_dense_fp32(int8):
    """A vocabulary of 3 chunks with a ragged tail, H = 1024, 700 rows in two token chunks (a ragged one),
    against torch fp32 on the GPU."""
    import smelb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    V, H, N = 2 * 16384 + 1000, 1024, 700
    W = (torch.randn(V, H, device=dev, generator=g) * 0.03).bfloat16()
    head = smelb.LMHead.from_weight(W, int8=int8, vocab_chunk=16384)
    h = torch.randn(N, H, device=dev, generator=g).bfloat16().requires_grad_(True)
    tgt = torch.randint(0, V, (N,), device=dev, generator=g)
    loss = smelb.chunked_ce(h, head, tgt, denom=N, token_chunk=512)
    loss.backward()
    Wf = head.rows(0, V, torch.float32)
    hr = h.detach().float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(hr @ Wf.t(), tgt)
    ref.backward()
    assert abs(float(loss) - float(ref)) < 1e-2
    rel = float((h.grad.float() - hr.grad).norm() / hr.grad.norm())
    assert rel < 2e-2 and _cos(h.grad, hr.grad) > 0.9999, rel
