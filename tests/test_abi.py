"""The C-ABI library: loads, exports every entry point include/smelb.h declares, and its struct matches the
binding. No GPU needed (no compute calls)."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "smelb.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|size_t|void|long long)\s+(smelb_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from smelb import _lib
    lib = _lib.load()
    names = declared()
    assert len(names) >= 12
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # every declared entry point also has a binding signature
    assert set(names) <= set(_lib.SIGNATURES)


def test_layer_struct_mirror_matches_c():
    from smelb import _lib
    assert _lib.load().smelb_moe_layer_size() == ctypes.sizeof(_lib.MoELayerStruct)


def test_version_and_error_text():
    from smelb import _lib
    assert _lib.load().smelb_version() >= 100
    assert isinstance(_lib.last_error(), str)


def test_null_pointer_is_an_error_not_a_crash():
    from smelb import _lib
    with pytest.raises(_lib.SmelbError, match="null pointer"):
        _lib.call("smelb_int4_dequant", None, None, None, None, 1, 64, 1, 0, None)


def test_cpu_tensors_are_rejected():
    """There is no CPU path: the API refuses CPU tensors instead of computing with torch."""
    import smelb
    q = torch.zeros(2, 32, dtype=torch.uint8)
    s = torch.ones(2, 1, dtype=torch.bfloat16)
    with pytest.raises(smelb.SmelbError):
        smelb.dequant_int4(q, s, s)
    with pytest.raises(smelb.SmelbError):
        smelb.quantize_int4(torch.randn(2, 64))
    with pytest.raises(smelb.SmelbError):
        smelb.route(torch.randn(4, 64, dtype=torch.bfloat16), torch.randn(8, 64, dtype=torch.bfloat16), 2)


def test_chunked_ce_workspace_sizes():
    """Workspace of smelb_chunked_ce: the bf16 logit tile of one (token chunk, vocabulary chunk), the fp32 state of
    every row, the gradient's fp32 partials and accumulators only when the gradient is formed, and a bf16 copy of
    one head chunk only for an int8 head."""
    from smelb import _lib
    ws = _lib.load().smelb_chunked_ce_workspace_bytes
    N, tc, H, vc = 4092, 1024, 2048, 32768
    full = ws(N, tc, H, vc, 0, 1)
    assert full >= tc * vc * 2 + 2 * N * H * 4 + 4 * tc * H * 4
    assert ws(N, tc, H, vc, 1, 1) - full == vc * H * 2           # the dequantised head chunk
    assert ws(N, tc, H, vc, 0, 0) < full - 2 * N * H * 4          # no accumulators without the gradient
    assert ws(N, 2 * tc, H, vc, 0, 1) > full                      # the logit tile grows with the token chunk
    assert ws(N, 4 * N, H, vc, 0, 1) == ws(N, N, H, vc, 0, 1)     # token chunks are capped at N rows
    assert ws(0, tc, H, vc, 0, 1) == 256                          # empty input: a minimal buffer
    assert _lib.load().smelb_lm_logits_workspace_bytes(N, H, vc, 1) >= N * vc * 2 + vc * H * 2


def test_ce_and_int8_argument_errors():
    """The CE and int8-row entry points reject bad arguments before launching anything."""
    from smelb import _lib
    with pytest.raises(_lib.SmelbError, match="null pointer"):
        _lib.call("smelb_chunked_ce", None, None, 4, 64, None, None, None, 100, 64, 64, 0.0, 1.0, None, None, None,
                  None, 0, None)
    fake = 1 << 20  # never dereferenced: the shape check fails first
    with pytest.raises(_lib.SmelbError, match="exactly one"):
        _lib.call("smelb_chunked_ce", fake, fake, 4, 64, fake, fake, fake, 100, 64, 64, 0.0, 1.0, fake, fake, None,
                  fake, 1 << 30, None)
    with pytest.raises(_lib.SmelbError, match="H=100"):
        _lib.call("smelb_chunked_ce", fake, fake, 4, 100, fake, None, None, 100, 64, 64, 0.0, 1.0, fake, fake, None,
                  fake, 1 << 30, None)
    with pytest.raises(_lib.SmelbError, match="softcap"):
        _lib.call("smelb_chunked_ce", fake, fake, 4, 64, fake, None, None, 100, 64, 64, -1.0, 1.0, fake, fake, None,
                  fake, 1 << 30, None)
    with pytest.raises(_lib.SmelbError, match="workspace"):
        _lib.call("smelb_chunked_ce", fake, fake, 4, 64, fake, None, None, 100, 64, 64, 0.0, 1.0, fake, fake, None,
                  fake, 16, None)
    with pytest.raises(_lib.SmelbError, match="null pointer"):
        _lib.call("smelb_int8_rows_quantize", None, 0, 4, 64, None, None, None)
    with pytest.raises(_lib.SmelbError, match="null pointer"):
        _lib.call("smelb_int8_rows_dequant", None, None, 4, 64, None, 0, None)
