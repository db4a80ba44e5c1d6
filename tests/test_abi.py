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
