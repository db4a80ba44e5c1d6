"""Layer weight sources (smelb/stream.py, smel/stream.py:16-114): the packed-key mapping of build_layer on the CPU,
and on the GPU a three-layer stack streamed from pinned host memory (two layers on the GPU at a time, forward order
then reverse order as the backward walks it) giving exactly the outputs of the resident layers."""
import pytest
import torch


def _packed(ex, W):
    t = dict(W)
    for k, v in ex.frozen.gu.items():
        t["experts.gate_up." + k] = v
    for k, v in ex.frozen.dn.items():
        t["experts.down." + k] = v
    if ex.sel_ids is not None:
        t["experts.sel.gate_up"], t["experts.sel.down"] = ex.sel_gate_up, ex.sel_down
        t["experts.sel.ids"] = ex.sel_ids.clone()
    return t


def test_build_layer_maps_packed_keys_cpu():
    import smelb
    from smelb.stream import build_layer
    E, N, K = 4, 128, 64
    t = {"experts.gate_up.q": torch.zeros(E, N, K // 2, dtype=torch.uint8),
         "experts.gate_up.scale": torch.ones(E, N, 1, dtype=torch.bfloat16),
         "experts.gate_up.zero": torch.zeros(E, N, 1, dtype=torch.bfloat16),
         "experts.down.q": torch.zeros(E, K, N // 4, dtype=torch.uint8),
         "experts.down.scale": torch.ones(E, K, 1, dtype=torch.bfloat16),
         "experts.down.zero": torch.zeros(E, K, 1, dtype=torch.bfloat16),
         "experts.sel.gate_up": torch.zeros(2, N, K, dtype=torch.bfloat16),
         "experts.sel.down": torch.zeros(2, K, N // 2, dtype=torch.bfloat16),
         "experts.sel.ids": torch.tensor([3, 1]),
         "mlp.gate.weight": torch.zeros(E, K, dtype=torch.bfloat16)}
    dense, ex = build_layer(t, act="gelu_tanh")
    assert set(dense) == {"mlp.gate.weight"}
    assert isinstance(ex.frozen, smelb.Int4Experts) and ex.frozen.num_experts == E
    assert ex.frozen.gu["q"] is t["experts.gate_up.q"] and ex.frozen.dn["zero"] is t["experts.down.zero"]
    assert ex.sel_ids.tolist() == [3, 1] and ex.act == "gelu_tanh"
    bf = {"mlp.experts.gate_up_proj": torch.zeros(E, N, K, dtype=torch.bfloat16),
          "mlp.experts.down_proj": torch.zeros(E, K, N // 2, dtype=torch.bfloat16)}
    dense, ex = build_layer(bf, sel_ids=[2])
    assert isinstance(ex.frozen, smelb.BF16Experts) and ex.sel_ids.tolist() == [2]
    assert ex.sel_gate_up.shape == (1, N, K)


@pytest.mark.gpu
def test_streamed_layers_equal_resident_layers():
    import smelb
    from smelb.stream import LayerSource
    from smelb.synth import qwen_layer
    dev = torch.device("cuda", 0)
    layers, ref_out, xs = {}, {}, {}
    for l in range(3):
        L = qwen_layer(T=96, H=256, E=16, K=4, I=128, S=128, n_sel=2, r=8, alpha=16.0, seed=10 + l, device=dev,
                       with_lora=False)
        xs[l] = L["x"]
        with torch.no_grad():
            ref_out[l] = smelb.moe_forward(L["x"], L["W"], L["ex"], 4, None)
        layers[l] = {k: v.cpu() for k, v in _packed(L["ex"], L["W"]).items()}
    src = LayerSource(layers, device=dev, max_on_gpu=2, timing=True)
    with torch.no_grad():
        order = [0, 1, 2, 2, 1, 0]
        for i, l in enumerate(order):
            dense, ex = src.get(l)
            if i + 1 < len(order):
                src.prefetch(order[i + 1])
            out = smelb.moe_forward(xs[l], dense, ex, 4, None)
            assert torch.equal(out, ref_out[l]), f"layer {l} (step {i})"
            assert len(src.cache) + len(src.pending) <= 2
    torch.cuda.synchronize()
    assert src.stats["loads"] >= 4 and src.stats["bytes"] > 0 and src.wait_ms() >= 0.0
    src.close()
    res = LayerSource(layers, device=dev, resident=True)
    assert res.stats["loads"] == 3
    with torch.no_grad():
        for l in (2, 0, 1):
            dense, ex = res.get(l)
            assert torch.equal(smelb.moe_forward(xs[l], dense, ex, 4, None), ref_out[l])
    assert res.stats["loads"] == 3
    assert smelb.read_status() == 0
