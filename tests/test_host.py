"""Host-side logic that needs no GPU: synthetic inputs, roofline arithmetic, dispatch-layout bookkeeping."""
import numpy as np

from oracle import moe_oracle as O


def test_packed_lengths_cover_tokens():
    from smelb.synth import packed_lengths
    lens, cu = packed_lengths(4092, seed=0)
    assert sum(lens) == 4092 and cu[-1] == 4092 and cu[0] == 0
    assert all(64 <= n for n in lens)
    assert max(lens[:-1]) <= 1024


def test_flops_per_token_qwen():
    from smelb.synth import flops_per_token
    f = flops_per_token(2048, 256, 8, 512, 512)
    base = 2 * 8 * 3 * 2048 * 512 + 2 * 3 * 2048 * 512 + 2 * 2048 * 256
    assert abs(base - 57.67e6) / 57.67e6 < 1e-3
    assert f > base


def test_bank_bytes_per_expert():
    from smelb.synth import int4_bank_bytes_per_expert
    assert int4_bank_bytes_per_expert(2048, 512) == 3 * 2048 * 512 // 2 + 3 * 2048 * 512 // 16


def test_dispatch_padded_handles_empty_and_all_selected():
    topi = np.array([[1, 2], [2, 1], [1, 2]])
    sel = np.ones(4, dtype=np.uint8)
    counts, gcounts, offsets, row_of, src_of = O.dispatch_padded(topi, 4, sel, pad=64)
    assert counts.tolist() == [0, 3, 3, 0]
    assert gcounts.tolist() == [0, 64, 64, 0]
    assert offsets.tolist() == [0, 0, 64, 128]
    assert row_of.tolist() == [0, 64, 65, 1, 2, 66]
