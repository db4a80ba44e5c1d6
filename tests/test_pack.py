"""The packed on-disk block (smelb/pack.py, smel/pack.py:8-46) against the reference's own output
(tests/golden/pack.pt, written by tests/golden/make_golden.py --only pack): safetensors round trip on the CPU;
pack_layer with the CUDA quantizer and the LoRA merges with the CUDA merge kernel on the GPU (bit-exact)."""
import pytest
import torch

NAMES = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")


def _same(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.view(torch.uint8) if a.dtype.is_floating_point
                                                                     else a, b.view(torch.uint8)
                                                                     if b.dtype.is_floating_point else b)


def test_packed_file_round_trip(golden, tmp_path):
    from smelb import pack
    d = golden("pack.pt")
    pack.save_layer(str(tmp_path), 7, d["packed"])
    assert (tmp_path / "layer_07.safetensors").exists()
    back = pack.load_layer(str(tmp_path), 7)
    assert set(back) == set(d["packed"])
    for k, v in d["packed"].items():
        assert _same(back[k], v), k


def test_merge_without_cuda_fails_loudly(golden):
    """There is no CPU merge: without a CUDA device the merge raises instead of computing on the host."""
    import smelb
    from smelb import pack
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    d = golden("pack.pt")
    t = d["t"]
    S, H = t["mlp.shared_expert.gate_proj.weight"].shape
    lsh = smelb.MLPLoRA(H, S, d["r"], d["alpha"])
    with pytest.raises(smelb.SmelbError):
        pack.merge_mlp(t["mlp.shared_expert.gate_proj.weight"].bfloat16(),
                       t["mlp.shared_expert.up_proj.weight"].bfloat16(),
                       t["mlp.shared_expert.down_proj.weight"].bfloat16(), lsh)


@pytest.mark.gpu
def test_merges_equal_reference(golden):
    """The CUDA merge (fp32 fma chain over the rank, one rounding) equals the reference's torch merge bit for bit,
    for CPU inputs (moved to the GPU and back) and CUDA inputs."""
    import smelb
    from smelb import pack
    d = golden("pack.pt")
    t, sel, r, alpha = d["t"], d["sel"], d["r"], d["alpha"]
    E, I2, H = t["mlp.experts.gate_up_proj"].shape
    S = t["mlp.shared_expert.gate_proj.weight"].shape[0]
    lex = smelb.ExpertsLoRA(sel, H, I2 // 2, r, alpha)
    lsh = smelb.MLPLoRA(H, S, r, alpha)
    with torch.no_grad():
        for n in NAMES:
            getattr(lex, n).copy_(d["lora_ex"][n])
            getattr(lsh, n).copy_(d["lora_sh"][n])
    gu, dn = pack.merge_experts(t["mlp.experts.gate_up_proj"].bfloat16(), t["mlp.experts.down_proj"].bfloat16(), lex)
    assert _same(gu, d["merged_gu"]) and _same(dn, d["merged_dn"])
    dev = torch.device("cuda", 0)
    gu2, dn2 = pack.merge_experts(t["mlp.experts.gate_up_proj"].bfloat16().to(dev),
                                  t["mlp.experts.down_proj"].bfloat16().to(dev), lex.to(dev))
    assert gu2.is_cuda and _same(gu2.cpu(), d["merged_gu"]) and _same(dn2.cpu(), d["merged_dn"])
    m = pack.merge_mlp(t["mlp.shared_expert.gate_proj.weight"].bfloat16(),
                       t["mlp.shared_expert.up_proj.weight"].bfloat16(),
                       t["mlp.shared_expert.down_proj.weight"].bfloat16(), lsh)
    for a, b in zip(m, d["merged_mlp"]):
        assert _same(a, b)


@pytest.mark.gpu
def test_pack_layer_on_gpu_equals_reference(golden):
    """Dense, integer and selected-expert tensors bit-exact; the int4 bank equal to the reference's except on
    near-ties of the quantizer's clip candidates (as the quantizer test allows)."""
    from smelb import pack
    d = golden("pack.pt")
    dev = torch.device("cuda", 0)
    t = {k: v.to(dev) for k, v in d["t"].items()}
    out = {k: v.cpu() for k, v in pack.pack_layer(t, d["sel"], 64).items()}
    ref = d["packed"]
    assert set(out) == set(ref)
    for k, v in ref.items():
        if not k.startswith(("experts.gate_up.", "experts.down.")):
            assert _same(out[k], v), k
    for name in ("gate_up", "down"):
        s_ok = out[f"experts.{name}.scale"].view(torch.int16) == ref[f"experts.{name}.scale"].view(torch.int16)
        z_ok = out[f"experts.{name}.zero"].view(torch.int16) == ref[f"experts.{name}.zero"].view(torch.int16)
        ok = (s_ok & z_ok).reshape(-1)
        assert ok.float().mean() > 0.99, name
        q, qr = out[f"experts.{name}.q"].reshape(ok.numel(), -1), ref[f"experts.{name}.q"].reshape(ok.numel(), -1)
        assert torch.equal(q[ok], qr[ok]), name
