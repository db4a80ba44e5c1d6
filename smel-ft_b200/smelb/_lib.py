"""ctypes binding of libsmelb.so (the C ABI declared in include/smelb.h).

The library is built in-tree (smel-ft_b200/build.py) and loaded from this directory. There is no fallback: every
public function of smelb raises SmelbError when the library is missing or when it is called on CPU tensors.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsmelb.so")

ACT = {"silu": 0, "gelu_tanh": 1}

F_ROUTER, F_ROUTED, F_SHARED, F_SHARED_GATE, F_SAVE, F_TOPV_FP32, F_RECOMPUTE = 1, 2, 4, 8, 16, 32, 64
F_EXT_DISPATCH = 128

ERRORS = {-1: "bad shape", -2: "bad dtype", -3: "workspace too small", -4: "device wait timed out",
          -5: "CUDA error", -6: "bad argument"}


class SmelbError(RuntimeError):
    """A smelb C-ABI call failed (or the CUDA library is unavailable)."""


_lib = None

c_i64, c_i32, c_f32, c_vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p

# field list of struct smelb_moe_layer, in declaration order (include/smelb.h)
_LAYER_FIELDS = [
    ("T", c_i64), ("H", c_i64), ("E", c_i64), ("K", c_i64), ("I", c_i64), ("S", c_i64), ("n_sel", c_i64),
    ("r_sel", c_i64), ("r_sh", c_i64), ("s_sel", c_f32), ("s_sh", c_f32), ("act", c_i32), ("flags", c_i32),
    ("max_rows", c_i64), ("stream", c_vp),
    ("x", c_vp), ("w_router", c_vp), ("w_sgate", c_vp), ("topv_in", c_vp), ("topi_in", c_vp), ("tok_count", c_vp),
    ("gu_q", c_vp), ("gu_sz", c_vp), ("dn_q", c_vp), ("dn_sz", c_vp),
    ("frozen_ids", c_vp), ("sel_ids", c_vp), ("sel_slots", c_vp), ("sel_mask", c_vp), ("sel_gu", c_vp),
    ("sel_dn", c_vp),
    ("A_gate", c_vp), ("B_gate", c_vp), ("A_up", c_vp), ("B_up", c_vp), ("A_down", c_vp), ("B_down", c_vp),
    ("sh_gu", c_vp), ("sh_dn", c_vp),
    ("shA_gate", c_vp), ("shB_gate", c_vp), ("shA_up", c_vp), ("shB_up", c_vp), ("shA_down", c_vp),
    ("shB_down", c_vp),
    ("out", c_vp), ("probs", c_vp), ("topv", c_vp), ("topi", c_vp), ("logits", c_vp), ("sgate_logit", c_vp),
    ("counts", c_vp), ("gcounts", c_vp), ("offsets", c_vp), ("row_of", c_vp), ("src_of", c_vp), ("total", c_vp),
    ("order", c_vp),
    ("xs", c_vp), ("h", c_vp), ("a", c_vp), ("y", c_vp), ("xa", c_vp), ("z", c_vp),
    ("sh_xa", c_vp), ("sh_h", c_vp), ("sh_a", c_vp), ("sh_z", c_vp), ("sh_y", c_vp),
    ("p_xa_w", c_vp), ("p_gu_ext", c_vp), ("p_z_w", c_vp), ("p_dn_ext", c_vp),
    ("sp_xa_w", c_vp), ("sp_gu_ext", c_vp), ("sp_z_w", c_vp), ("sp_dn_ext", c_vp),
    ("g", c_vp), ("dx", c_vp), ("dy", c_vp), ("dh", c_vp), ("dxs", c_vp), ("dz", c_vp), ("dxa", c_vp),
    ("dtopv", c_vp), ("dlogits", c_vp), ("dx_router", c_vp),
    ("sh_dy", c_vp), ("sh_dh", c_vp), ("sh_dx", c_vp), ("sh_dz", c_vp), ("sh_dxa", c_vp), ("dgl", c_vp),
    ("p_dz_w", c_vp), ("p_da_ext", c_vp), ("p_dxa_w", c_vp), ("p_dx_ext", c_vp),
    ("sp_dz_w", c_vp), ("sp_da_ext", c_vp), ("sp_dxa_w", c_vp), ("sp_dx_ext", c_vp),
    ("gA_gate", c_vp), ("gB_gate", c_vp), ("gA_up", c_vp), ("gB_up", c_vp), ("gA_down", c_vp), ("gB_down", c_vp),
    ("gshA_gate", c_vp), ("gshB_gate", c_vp), ("gshA_up", c_vp), ("gshB_up", c_vp), ("gshA_down", c_vp),
    ("gshB_down", c_vp),
    ("dprobs", c_vp), ("fz_gu", c_vp), ("fz_dn", c_vp), ("act_sh", c_i32), ("reserved", c_i32),
    ("per_expert_scale", c_vp), ("split_counts", c_vp),
]


class MoELayerStruct(ctypes.Structure):
    _fields_ = _LAYER_FIELDS


# exported symbol -> (restype, argtypes)
SIGNATURES = {
    "smelb_version": (c_i32, []),
    "smelb_last_error": (c_i32, [ctypes.c_char_p, ctypes.c_size_t]),
    "smelb_read_status": (c_i32, [c_i32, ctypes.POINTER(c_i32), c_i32]),
    "smelb_set_device": (c_i32, [c_i32]),
    "smelb_read_status_detail": (c_i32, [c_i32, ctypes.POINTER(c_i32), c_i32]),
    "smelb_int4_dequant": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_vp]),
    "smelb_int4_pack_sz": (c_i32, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "smelb_int4_quantize": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_vp, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "smelb_router_topk": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_i32, c_vp, c_vp, c_vp]),
    "smelb_router_bwd": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "smelb_dispatch_plan": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                    c_vp, c_vp]),
    "smelb_dispatch_plan_ws": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                       c_vp, c_i64, c_vp]),
    "smelb_gather_rows": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_vp, c_vp]),
    "smelb_combine_fwd": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "smelb_rmsnorm_fwd": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_vp, ctypes.c_float, ctypes.c_float, c_i64, c_i64, c_vp,
                                  c_vp, c_vp, c_vp]),
    "smelb_rmsnorm_bwd": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_vp, ctypes.c_float, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp]),
    "smelb_combine_bwd": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "smelb_gather_rows_bwd": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "smelb_frozen_experts_fwd": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i32,
                                         c_vp, c_vp, c_vp, c_vp]),
    "smelb_frozen_experts_bwd": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp,
                                         c_i32, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "smelb_frozen_experts_fwd_noalloc": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp,
                                                 c_i32, c_vp, c_vp, c_vp]),
    "smelb_frozen_experts_fwd_noalloc_status": (c_i32, [c_i32, ctypes.POINTER(c_i32), c_i32]),
    "smelb_frozen_experts_bf16_fwd": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_i32, c_vp, c_vp,
                                              c_vp, c_vp]),
    "smelb_frozen_experts_bf16_bwd": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_i32, c_vp,
                                              c_vp, c_vp, c_vp, c_vp]),
    "smelb_int4_dequant_stepwise": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_vp]),
    "smelb_lora_merge": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_i64, c_f32, c_vp, c_vp]),
    "smelb_lora_linear_workspace_bytes": (c_i64, [c_i64, c_i64, c_i64]),
    "smelb_lora_linear_fwd": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_f32, c_vp,
                                      c_vp, c_vp, c_i64, c_vp]),
    "smelb_lora_linear_bwd": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_f32,
                                      c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "smelb_ep_region_bytes": (c_i64, [c_i64, c_i64, c_i64, c_i64]),
    "smelb_ep_region_alloc": (c_i32, [c_i64, c_vp, c_vp]),
    "smelb_ep_region_open": (c_i32, [c_vp, c_vp]),
    "smelb_ep_region_close": (c_i32, [c_vp]),
    "smelb_ep_region_free": (c_i32, [c_vp]),
    "smelb_ep_sync": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_vp]),
    "smelb_ep_plan": (c_i32, [c_vp, c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp,
                              c_vp, c_vp]),
    "smelb_ep_pack_rows": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_vp]),
    "smelb_ep_recv_plan": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp,
                                   c_vp, c_vp, c_vp]),
    "smelb_ep_pull_rows": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp]),
    "smelb_ep_gather": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "smelb_ep_return": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64,
                                c_i32, c_vp]),
    "smelb_ep_dy": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "smelb_ep_collect": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32,
                                 c_vp, c_vp, c_vp, c_vp, c_i32, c_vp, c_vp]),
    "smelb_int8_rows_quantize": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "smelb_int8_rows_dequant": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_vp, c_i32, c_vp]),
    "smelb_chunked_ce_workspace_bytes": (c_i64, [c_i64, c_i64, c_i64, c_i64, c_i32, c_i32]),
    "smelb_chunked_ce": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_f32, c_f32, c_vp,
                                 c_vp, c_vp, c_vp, c_i64, c_vp]),
    "smelb_lm_logits_workspace_bytes": (c_i64, [c_i64, c_i64, c_i64, c_i32]),
    "smelb_lm_logits": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_f32, c_vp, c_vp, c_i64, c_vp]),
    "smelb_moe_layer_size": (ctypes.c_size_t, []),
    "smelb_launch_count": (ctypes.c_longlong, []),
    "smelb_gemm_timing": (c_i32, [c_i32]),
    "smelb_set_gemv_rows": (c_i64, [c_i64]),
    "smelb_gemm_timing_read": (c_i32, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong)]),
    "smelb_moe_layer_fwd": (c_i32, [ctypes.POINTER(MoELayerStruct)]),
    "smelb_moe_layer_bwd": (c_i32, [ctypes.POINTER(MoELayerStruct)]),
}


def load(path=LIB_PATH):
    """Load the library (once) and declare the C signatures. Raises SmelbError if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise SmelbError(f"libsmelb.so not found at {path}; build it with `python smel-ft_b200/build.py`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _lib = lib
    return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().smelb_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def call(name, *args):
    """Call an entry point on torch's current device and raise SmelbError with the library's message on a non-zero
    status."""
    lib = load()
    if torch.cuda.is_available():
        lib.smelb_set_device(torch.cuda.current_device())
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise SmelbError(f"{name}: {ERRORS.get(rc, rc)}: {last_error()}")


def read_status(device=None, reset=True) -> int:
    """Synchronize `device` and return its device status word (0 = no device-side wait gave up)."""
    dev = torch.cuda.current_device() if device is None else device
    v = c_i32(0)
    call("smelb_read_status", dev, ctypes.byref(v), 1 if reset else 0)
    return v.value


def launch_count() -> int:
    """Kernels launched by libsmelb so far."""
    return int(load().smelb_launch_count())


def set_gemv_rows(rows: int) -> int:
    """Dispatch rows at or below which the forward's frozen int4 experts run as the dequant-GEMV (0: never); within
    it, calls of at most 6 tokens also take the router / shared-gate logits and the shared expert (without LoRA) as
    dense GEMVs. Returns the previous value."""
    return int(load().smelb_set_gemv_rows(int(rows)))


def gemm_timing(enable: bool):
    call("smelb_gemm_timing", 1 if enable else 0)


def gemm_timing_read():
    """(summed ms, launches) of the expert-GEMM launches recorded since the last read (synchronizes)."""
    ms, n = ctypes.c_double(0), ctypes.c_longlong(0)
    call("smelb_gemm_timing_read", ctypes.byref(ms), ctypes.byref(n))
    return ms.value, n.value


def read_status_detail(device=None, reset=True):
    """(code, block, tile, k-block) of the first device-side failure (code 0 = none). Synchronizes."""
    dev = torch.cuda.current_device() if device is None else device
    w = (c_i32 * 4)()
    call("smelb_read_status_detail", dev, w, 1 if reset else 0)
    return tuple(w)


def ptr(t):
    """Device pointer of a CUDA tensor (None -> NULL). CPU tensors are rejected: there is no CPU path."""
    if t is None:
        return None
    if not t.is_cuda:
        raise SmelbError("smelb runs on CUDA tensors only (got a CPU tensor)")
    return t.data_ptr()


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream
