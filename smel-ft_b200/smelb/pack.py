"""The packed on-disk block of SMEL FT: one safetensors file per layer, `layer_XX.safetensors`, holding the layer's
dense tensors, its frozen expert bank in the int4 group format and bf16 copies of the selected experts; plus the merge
of trained LoRA deltas into bf16 weights. The file format and the merge arithmetic are the reference's
(smel/pack.py:8-46); the work runs on the GPU: the bank through the CUDA int4 quantizer, the merges through one
`smelb_lora_merge` kernel per weight block (the rank-r delta and the add fused, one rounding).

Keys (names relative to the layer, so files written by either side load in the other):
  experts.gate_up.{q,scale,zero}, experts.down.{q,scale,zero}      int4 bank (uint8 nibbles, bf16 scale / zero)
  experts.sel.ids (int64), experts.sel.gate_up, experts.sel.down    selected experts (bf16 copies)
  every tensor not under mlp.experts.                               bf16, except integer tensors and A_log / dt_bias
                                                                    (kept as stored)
"""
import os

import torch

from . import _lib
from .quant import quantize_int4

# checkpoint names of the fused expert bank, by packed part name
BANK = {"gate_up": "mlp.experts.gate_up_proj", "down": "mlp.experts.down_proj"}
BANK_PREFIX = "mlp.experts."
# floating-point tensors the packed file keeps in their stored dtype (DeltaNet's A_log and dt_bias)
KEEP_AS_STORED = ("A_log", "dt_bias")


def layer_path(packed_dir: str, l: int) -> str:
    return os.path.join(packed_dir, f"layer_{l:02d}.safetensors")


def _packed_dense(name: str, t: torch.Tensor, dtype) -> torch.Tensor:
    as_stored = not t.is_floating_point() or name.endswith(KEEP_AS_STORED)
    return (t if as_stored else t.to(dtype)).contiguous()


def _packed_bank(bank: dict, group: int) -> dict:
    """experts.{part}.{q,scale,zero} straight from the quantizer's outputs (one CUDA pass per matrix)."""
    return {f"experts.{part}.{field}": v for part, w in bank.items() for field, v in quantize_int4(w, group).items()}


def _packed_selected(bank: dict, sel_ids, dtype) -> dict:
    ids = torch.as_tensor(list(sel_ids), dtype=torch.long)
    out = {"experts.sel.ids": ids}
    for part, w in bank.items():
        out[f"experts.sel.{part}"] = w.index_select(0, ids.to(w.device)).to(dtype).contiguous()
    return out


def pack_layer(t: dict, sel_ids=None, group: int = 64, dtype=torch.bfloat16) -> dict:
    """The packed tensors of one checkpoint layer `t` (names relative to the layer), whose fused bank
    mlp.experts.gate_up_proj [E, 2I, H] / mlp.experts.down_proj [E, H, I] lies on a CUDA device (smel/pack.py:8-25).
    Other mlp.experts.* tensors are not packed."""
    bank = {part: t[name] for part, name in BANK.items()}
    packed = {name: _packed_dense(name, v, dtype) for name, v in t.items() if not name.startswith(BANK_PREFIX)}
    if sel_ids is not None and len(sel_ids):
        packed.update(_packed_selected(bank, sel_ids, dtype))
    packed.update(_packed_bank(bank, group))
    return packed


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


# ------------------------------------------------------------------------------------------ LoRA merges
def _on_gpu(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t
    if not torch.cuda.is_available():
        raise _lib.SmelbError("LoRA merge: smelb merges on the GPU and no CUDA device is available")
    return t.cuda()


def _merge_block(w: torch.Tensor, B: torch.Tensor, A: torch.Tensor, scale: float):
    """w (a contiguous bf16 / fp32 CUDA block [rows, cols]) += (scale B) @ A in place, one rounding per element."""
    if w.dtype not in (torch.bfloat16, torch.float32) or not w.is_contiguous():
        raise _lib.SmelbError(f"LoRA merge: expects a contiguous bf16 or fp32 weight, got {w.dtype}")
    B32 = B.detach().to(w.device, torch.float32).contiguous()
    A32 = A.detach().to(w.device, torch.float32).contiguous()
    rows, cols = w.shape
    _lib.call("smelb_lora_merge", _lib.ptr(w), 1 if w.dtype == torch.float32 else 0, rows, cols, _lib.ptr(B32),
              _lib.ptr(A32), A32.shape[0], float(scale), _lib.ptr(w), _lib.stream_ptr(w.device))


@torch.no_grad()
def merge_experts(gate_up: torch.Tensor, down: torch.Tensor, lora) -> tuple:
    """Copies of the fused expert tensors (gate_up [E, 2I, H], down [E, H, I]) with the LoRA deltas of the selected
    experts merged in: for slot j of expert e, gate rows += s B_gate[j] A_gate[j], up rows += s B_up[j] A_up[j],
    down += s B_down[j] A_down[j] (smel/pack.py:28-39). Returned on the inputs' device."""
    home = gate_up.device
    gu, dn = _on_gpu(gate_up).clone(), _on_gpu(down).clone()
    I = dn.shape[2]
    for j, e in enumerate(lora.expert_ids.tolist()):
        for block, name in ((gu[e, :I], "gate"), (gu[e, I:], "up"), (dn[e], "down")):
            _merge_block(block, getattr(lora, "B_" + name)[j], getattr(lora, "A_" + name)[j], lora.scale)
    return gu.to(home), dn.to(home)


@torch.no_grad()
def merge_mlp(gate_w, up_w, down_w, lora) -> tuple:
    """A gated MLP's three weights with its LoRA deltas merged in (smel/pack.py:42-46), on the inputs' device."""
    home = gate_w.device
    out = []
    for w, name in ((gate_w, "gate"), (up_w, "up"), (down_w, "down")):
        m = _on_gpu(w).clone()
        _merge_block(m, getattr(lora, "B_" + name), getattr(lora, "A_" + name), lora.scale)
        out.append(m.to(home))
    return tuple(out)
