"""Small-token path: the frozen int4 experts as a dequant-GEMV (csrc/gemv.cu) when a call has few dispatch rows
(smelb.set_gemv_rows; by default T*K <= 512 rows take it). Parity against the oracle at 1 to 128 tokens, uniform
and Zipf routing (a hot expert then holds more rows than one token tile and takes several passes), with the
reference layer's expert choices forced as in the other layer tests; the training forward's saved pre-activations
through the backward; and the GEMV against the tile engine at the config-4 shape (Qwen layer, all 256 experts
int4). Tolerance as the other layer tests: max relative error 2e-2, cosine 0.9999 (the GEMV applies each group's
(scale, zero) to fp32 sums instead of rounding every weight to bf16 first, so it and the tile engine agree far closer
than that: 1e-2 / 0.99995)."""
import pytest
import torch

from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
REL, COS = 2e-2, 0.9999
NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")


class _Bank:
    """The oracle's view of an int4 bank: one expert dequantized on the CPU on first access."""

    def __init__(self, d, dtype):
        self.q, self.s, self.z = d["q"].cpu(), d["scale"].cpu(), d["zero"].cpu()
        self.shape = (self.q.shape[0], self.q.shape[1], self.q.shape[2] * 2)
        self.dtype, self.cache = dtype, {}

    def __getitem__(self, e):
        if e not in self.cache:
            self.cache[e] = O.dequant_int4(self.q[e], self.s[e], self.z[e]).to(self.dtype)
        return self.cache[e]


def _close(items, rel=REL, cos=COS):
    bad = []
    for what, a, b in items:
        e, c = O.rel_err(a.float().cpu(), b.float().cpu()), O.cosine(a.float().cpu(), b.float().cpu())
        print(f"{what:>18s}: rel err {e:.3e} cosine {c:.7f}")
        if not (e <= rel and c >= cos):
            bad.append(f"{what}: rel err {e:.3e}, cosine {c:.6f}")
    assert not bad, "; ".join(bad)


@pytest.fixture
def gemv_rows():
    """Sets the GEMV row limit for one test and puts the previous value back."""
    import smelb
    prev = smelb.set_gemv_rows(4096)
    smelb.set_gemv_rows(prev)
    yield smelb.set_gemv_rows
    smelb.set_gemv_rows(prev)


def _layer(T, E, routing, seed, **kw):
    from smelb.synth import qwen_layer
    args = dict(T=T, H=2048, E=E, K=8, I=512, S=512, n_sel=0, with_lora=False, seed=seed, device="cuda:0",
                uniform=routing == "uniform", zipf_s=1.2, tau=1.0)
    args.update(kw)
    return qwen_layer(**args)


@pytest.mark.parametrize("routing", ["uniform", "zipf"])
@pytest.mark.parametrize("T", [1, 5, 16, 33, 128])
def test_small_token_forward_vs_oracle(T, routing, gemv_rows):
    import smelb
    gemv_rows(1 << 30)
    L = _layer(T, 64, routing, seed=10 + T)
    x, W, ex = L["x"], L["W"], L["ex"]
    rec = {}
    with torch.no_grad():
        out = smelb.moe_forward(x, W, ex, 8, None, stats=lambda p, v, i: rec.update(i=i))
    counts = torch.bincount(rec["i"].reshape(-1), minlength=64)
    print(f"T={T} {routing}: {int((counts > 0).sum())} experts touched, hottest {int(counts.max())} rows")
    dt = torch.float32
    ref, _, _, _ = O.moe_layer(x.cpu().to(dt), {k: v.cpu().to(dt) for k, v in W.items()}, _Bank(ex.frozen.gu, dt),
                               _Bank(ex.frozen.dn, dt), 8, act_name=ex.act, topi=rec["i"].cpu())
    _close([("out", out, ref)])
    assert smelb.read_status() == 0


@pytest.mark.parametrize("T", [24, 200])
def test_small_token_training_step_vs_oracle(T, gemv_rows):
    """Forward with the pre-activations saved by the GEMV epilogue (and with them recomputed instead), backward on
    the engine: out, dX and every LoRA gradient (the selected experts and the shared expert) against the oracle. At
    200 tokens (1600 dispatch rows, Zipf routing) the experts with more than 16 rows stay on the tile engine and the
    rest take the GEMV, in the forward and in the backward's recompute alike."""
    import smelb
    from smelb.synth import qwen_layer
    gemv_rows(1 << 30)
    L = qwen_layer(T=T, H=1024, E=48, K=8, I=256, S=256, n_sel=6, r=16, seed=21, device="cuda:0")
    meta, ex, lora = L["meta"], L["ex"], L["lora"]
    gy = torch.randn(L["x"].shape, generator=torch.Generator(device="cuda:0").manual_seed(3),
                     device="cuda:0").bfloat16()
    results = []
    for save in (True, False):
        prev = smelb.set_save_preactivations(save)
        try:
            for p in lora.parameters():
                p.grad = None
            x = L["x"].clone().requires_grad_(True)
            rec = {}
            out = smelb.moe_forward(x, L["W"], ex, 8, lora, stats=lambda p, v, i: rec.update(i=i))
            out.backward(gy)
        finally:
            smelb.set_save_preactivations(prev)
        results.append((out.detach(), x.grad, {n: getattr(lora.experts, n).grad.clone() for n in NAMES},
                        {n: getattr(lora.shared, n).grad.clone() for n in NAMES}, rec["i"].cpu()))
    out, dx, g_ex, g_sh, topi = results[0]
    counts = torch.bincount(topi.reshape(-1), minlength=48)
    print(f"T={T}: hottest expert {int(counts.max())} rows, {int((counts > 16).sum())} above 16")
    assert torch.equal(out, results[1][0]) and torch.equal(dx, results[1][1])
    dt = torch.float64
    x64 = L["x"].cpu().to(dt).requires_grad_(True)
    lex = {n: getattr(lora.experts, n).detach().cpu().to(dt).requires_grad_(True) for n in NAMES}
    lsh = {n: getattr(lora.shared, n).detach().cpu().to(dt).requires_grad_(True) for n in NAMES}
    s = lora.experts.scale
    ref, _, _, _ = O.moe_layer(x64, {k: v.cpu().to(dt) for k, v in L["W"].items()}, _Bank(ex.frozen.gu, dt),
                               _Bank(ex.frozen.dn, dt), 8, meta["selected"], ex.sel_gate_up.cpu().to(dt),
                               ex.sel_down.cpu().to(dt), {**lex, "scale": s}, {**lsh, "scale": s}, act_name=ex.act,
                               topi=topi)
    ref.backward(gy.cpu().to(dt))
    _close([("out", out, ref), ("dx", dx, x64.grad)] + [("experts " + n, g_ex[n], lex[n].grad) for n in NAMES] +
           [("shared " + n, g_sh[n], lsh[n].grad) for n in NAMES])
    for n in NAMES:
        assert torch.equal(results[1][2][n], g_ex[n]) and torch.equal(results[1][3][n], g_sh[n]), n
    assert smelb.read_status() == 0


@pytest.mark.parametrize("T", [1, 4, 6])
def test_small_token_shared_gemv_training_vs_oracle(T, gemv_rows):
    """At up to 6 tokens without LoRA the shared expert's projections run as dense GEMVs (csrc/dense.cu) in the
    forward and in the backward's recompute of its pre-activations: out and dX with the pre-activations saved and
    recomputed are identical, and both match the oracle (the tile engine run of the same step within 1e-2)."""
    import smelb
    gemv_rows(1 << 30)
    L = _layer(T, 64, "zipf", seed=30 + T)
    gy = torch.randn(L["x"].shape, generator=torch.Generator(device="cuda:0").manual_seed(5),
                     device="cuda:0").bfloat16()
    runs = []
    for rows, save in ((1 << 30, True), (1 << 30, False), (0, True)):
        gemv_rows(rows)
        prev = smelb.set_save_preactivations(save)
        try:
            x = L["x"].clone().requires_grad_(True)
            rec = {}
            out = smelb.moe_forward(x, L["W"], L["ex"], 8, None, stats=lambda p, v, i: rec.update(i=i))
            out.backward(gy)
        finally:
            smelb.set_save_preactivations(prev)
        runs.append((out.detach(), x.grad, rec["i"].cpu()))
    (out, dx, topi), (out_r, dx_r, _), (out_e, dx_e, topi_e) = runs
    assert torch.equal(out, out_r) and torch.equal(dx, dx_r)
    if torch.equal(topi, topi_e):
        _close([("out gemv vs engine", out, out_e), ("dx gemv vs engine", dx, dx_e)], rel=1e-2, cos=0.99995)
    dt = torch.float64
    x64 = L["x"].cpu().to(dt).requires_grad_(True)
    ex = L["ex"]
    ref, _, _, _ = O.moe_layer(x64, {k: v.cpu().to(dt) for k, v in L["W"].items()}, _Bank(ex.frozen.gu, dt),
                               _Bank(ex.frozen.dn, dt), 8, act_name=ex.act, topi=topi)
    ref.backward(gy.cpu().to(dt))
    _close([("out", out, ref), ("dx", dx, x64.grad)])
    assert smelb.read_status() == 0


@pytest.mark.parametrize("T", [1, 4, 16, 128, 1024])
def test_gemv_matches_tile_engine_config4(T, gemv_rows):
    """The small-token paths against the tile engine at the config-4 shape. Up to 6 tokens the router logits come from
    the dense GEMV as well; should a near-tie of the bf16 logits then resolve to another expert set, each path is
    checked against the oracle on its own choices instead."""
    import smelb
    L = _layer(T, 256, "uniform", seed=4)
    outs, tops = [], []
    for rows in (1 << 30, 0):
        gemv_rows(rows)
        rec = {}
        with torch.no_grad():
            outs.append(smelb.moe_forward(L["x"], L["W"], L["ex"], 8, None, stats=lambda p, v, i: rec.update(i=i)))
        tops.append(rec["i"].cpu())
    if torch.equal(tops[0], tops[1]):
        _close([("gemv vs engine", outs[0], outs[1])], rel=1e-2, cos=0.99995)
    else:
        dt, ex = torch.float32, L["ex"]
        for out, topi in zip(outs, tops):
            ref, _, _, _ = O.moe_layer(L["x"].cpu().to(dt), {k: v.cpu().to(dt) for k, v in L["W"].items()},
                                       _Bank(ex.frozen.gu, dt), _Bank(ex.frozen.dn, dt), 8, act_name=ex.act, topi=topi)
            _close([("out vs oracle", out, ref)])
    assert smelb.read_status() == 0


@pytest.mark.parametrize("act,H,I", [("silu", 1024, 192), ("gelu_tanh", 1024, 192), ("silu", 384, 128)])
def test_frozen_experts_fn_gemv_matches_engine(act, H, I, gemv_rows):
    """FrozenExpertsFn over expert-grouped rows without offsets (empty experts, one expert of 300 rows taking
    several token passes): the GEMV forward against the tile engine's, then the oracle. The shapes take each staging
    width of the packed rows: 128-byte boxes (H = 1024), 32-byte (I = 192) and 64-byte (H = 384, I = 128)."""
    import smelb
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(2)
    E = 8
    counts = [0, 5, 300, 17, 64, 1, 0, 9]
    bank = smelb.Int4Experts.from_bf16((torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.05).bfloat16(),
                                       (torch.randn(E, H, I, generator=g, device=dev) * 0.05).bfloat16())
    xs = torch.randn(sum(counts), H, generator=g, device=dev).bfloat16()
    ys = []
    for rows in (1 << 30, 0):
        gemv_rows(rows)
        with torch.no_grad():
            ys.append(smelb.FrozenExpertsFn.apply(xs, counts, bank, 32, act))
    gu = _Bank(bank.gu, torch.float64)
    dn = _Bank(bank.dn, torch.float64)
    ref = O.frozen_experts(xs.cpu().double(), counts, torch.stack([gu[e] for e in range(E)]),
                           torch.stack([dn[e] for e in range(E)]), act)
    _close([("gemv vs engine", ys[0], ys[1])], rel=1e-2, cos=0.99995)
    _close([("gemv vs oracle", ys[0], ref)])
    assert smelb.read_status() == 0
