"""The packed on-disk block of SMEL FT (smel/pack.py:1-62): one safetensors file per layer, `layer_XX.safetensors`,
holding the dense tensors in bf16, the frozen experts in the int4 group format and the selected experts as bf16
copies, plus the exact merge of LoRA deltas into bf16 weights.

Keys (names relative to the layer, as the reference writes them, so files written by either side load in the other):
  experts.gate_up.{q,scale,zero}, experts.down.{q,scale,zero}   int4 bank (uint8 nibbles, bf16 scale / zero)
  experts.sel.ids (int64), experts.sel.gate_up, experts.sel.down   selected experts (bf16)
  every other tensor                                              as stored, in bf16 unless it is an integer tensor
                                                                  or an A_log / dt_bias (kept as they are)
The int4 banks are quantized on the GPU (smelb.quant.quantize_int4, the CUDA quantizer for group 64).
"""
import os

import torch

from .quant import quantize_int4


def layer_path(packed_dir: str, l: int) -> str:
    return os.path.join(packed_dir, f"layer_{l:02d}.safetensors")


def pack_layer(t: dict, sel_ids=None, group: int = 64, dtype=torch.bfloat16) -> dict:
    """smel/pack.py:8-25. t: the tensors of one layer as stored in the checkpoint (names relative to the layer),
    with the fused bank `mlp.experts.gate_up_proj` [E, 2I, H] and `mlp.experts.down_proj` [E, H, I] on a CUDA
    device. Returns the packed dict (tensors on the bank's device)."""
    out = {}
    for k, v in t.items():
        if k.startswith("mlp.experts."):
            continue
        keep = k.endswith(("A_log", "dt_bias")) or not v.is_floating_point()
        out[k] = v.contiguous() if keep else v.to(dtype).contiguous()
    gu, dn = t["mlp.experts.gate_up_proj"], t["mlp.experts.down_proj"]
    if sel_ids is not None and len(sel_ids):
        ids = torch.as_tensor(list(sel_ids), dtype=torch.long)
        out["experts.sel.ids"] = ids
        out["experts.sel.gate_up"] = gu[ids.to(gu.device)].to(dtype).contiguous()
        out["experts.sel.down"] = dn[ids.to(dn.device)].to(dtype).contiguous()
    for name, w in (("gate_up", gu), ("down", dn)):
        for kk, vv in quantize_int4(w, group).items():
            out[f"experts.{name}.{kk}"] = vv
    return out


def save_layer(packed_dir: str, l: int, packed: dict):
    """Write one packed layer as `layer_XX.safetensors` (tensors are moved to the CPU)."""
    from safetensors.torch import save_file
    os.makedirs(packed_dir, exist_ok=True)
    save_file({k: v.detach().contiguous().cpu() for k, v in packed.items()}, layer_path(packed_dir, l))


def load_layer(packed_dir: str, l: int, pin: bool = False) -> dict:
    """Read `layer_XX.safetensors` into CPU tensors (pinned with pin=True, ready for smelb.stream.LayerSource)."""
    from safetensors import safe_open
    out = {}
    with safe_open(layer_path(packed_dir, l), "pt") as f:
        for k in f.keys():
            v = f.get_tensor(k)
            out[k] = v.pin_memory() if pin else v
    return out


@torch.no_grad()
def merge_experts(gate_up: torch.Tensor, down: torch.Tensor, lora) -> tuple:
    """smel/pack.py:28-39: copies of the fused expert tensors with the LoRA deltas of the selected experts added
    (fp32 math, one rounding to the tensors' dtype)."""
    gu, dn = gate_up.clone(), down.clone()
    I = dn.shape[2]
    for j, e in enumerate(lora.expert_ids.tolist()):
        dg, du, dd = (x.to(gu.device) for x in lora.delta(j))
        gu[e, :I] = (gu[e, :I].float() + dg).to(gu.dtype)
        gu[e, I:] = (gu[e, I:].float() + du).to(gu.dtype)
        dn[e] = (dn[e].float() + dd).to(dn.dtype)
    return gu, dn


@torch.no_grad()
def merge_mlp(gate_w, up_w, down_w, lora) -> tuple:
    """smel/pack.py:42-46: a gated MLP's three weights with its LoRA deltas added (fp32 math, one rounding)."""
    dg, du, dd = (x.to(gate_w.device) for x in lora.delta())
    return ((gate_w.float() + dg).to(gate_w.dtype), (up_w.float() + du).to(up_w.dtype),
            (down_w.float() + dd).to(down_w.dtype))
