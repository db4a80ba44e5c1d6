"""smelb: the SMEL FT MoE expert layer (smel/moe.py, smel/quant.py int4 group-64, smel/lora.py) on B200 (sm_100a).

Drop-in names for the reference modules:
    smel.moe  -> smelb.moe   (BF16Experts, Int4Experts, LayerExperts, FrozenExpertsFn, route, route_gemma4,
                              routed_experts, mlp_lora, shared_mlp, moe_forward)
    smel.norm / layer_runner norms -> smelb.norm (rmsnorm, add_rmsnorm); the Gemma 4 MoE block of
                              layer_runner.py:249-261 -> smelb.moe.moe_block_gemma4
    smel.quant-> smelb.quant (quantize_int4, dequant_int4, dequant_int4_torch, quantize_int8_rows,
                              dequant_int8_rows, rel_err)
    smel.loss -> smelb.loss  (LMHead, chunked_ce)
    smel.lora -> smelb.lora  (ExpertsLoRA, MLPLoRA, LayerLoRA, BlockLoRA, lora_linear, lora_gate_up)
All compute runs in libsmelb.so (hand-written CUDA for sm_100a) through the C ABI in include/smelb.h.
"""
from . import _lib
from ._lib import SmelbError, read_status, set_gemv_rows
from .loss import LMHead, chunked_ce
from .lora import BlockLoRA, ExpertsLoRA, LayerLoRA, MLPLoRA, lora_gate_up, lora_linear
from .moe import (BF16Experts, FrozenExpertsFn, Int4Experts, LayerExperts, mlp_lora, moe_block_gemma4, moe_forward,
                  route, route_gemma4, routed_experts, set_save_preactivations, shared_mlp)
from .norm import add_rmsnorm, rmsnorm
from .quant import dequant_int4, dequant_int4_torch, dequant_int8_rows, quantize_int4, quantize_int8_rows, rel_err

__all__ = ["BF16Experts", "BlockLoRA", "ExpertsLoRA", "FrozenExpertsFn", "Int4Experts", "LMHead", "LayerExperts",
           "LayerLoRA", "MLPLoRA", "SmelbError", "add_rmsnorm", "chunked_ce", "dequant_int4", "dequant_int4_torch",
           "dequant_int8_rows", "lora_gate_up", "lora_linear", "mlp_lora", "moe_block_gemma4", "moe_forward",
           "quantize_int4", "quantize_int8_rows", "read_status", "rel_err", "rmsnorm", "route", "route_gemma4",
           "routed_experts", "set_gemv_rows", "set_save_preactivations", "shared_mlp"]


def load_library():
    """Load libsmelb.so (raises SmelbError when it has not been built)."""
    return _lib.load()
