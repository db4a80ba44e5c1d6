"""LoRA parameters of the selected routed experts and of the shared expert / dense MLP (smel/lora.py:1-125).

Parameter names, shapes and initialisation follow the reference so adapters load unchanged:
  ExpertsLoRA (k slots): A_gate/A_up [k, r, H], B_gate/B_up [k, I, r], A_down [k, r, I], B_down [k, H, r]
  MLPLoRA:               A_gate/A_up [r, H],    B_gate/B_up [I, r],    A_down [r, I],    B_down [H, r]
A is initialised like PEFT (kaiming_uniform_(a=sqrt(5)) per [r, in] matrix), B with zeros, scale = alpha / r.
"""
import json
import math
import os

import torch
from torch import nn


def _init_a(t: torch.Tensor):
    for m in t.reshape(-1, *t.shape[-2:]):
        nn.init.kaiming_uniform_(m, a=math.sqrt(5))


class ExpertsLoRA(nn.Module):
    """LoRA for k selected experts of one layer; slot j belongs to global expert id expert_ids[j]."""

    def __init__(self, expert_ids, hidden: int, inter: int, r: int = 16, alpha: float = 32.0):
        super().__init__()
        k = len(expert_ids)
        self.register_buffer("expert_ids", torch.as_tensor(list(expert_ids), dtype=torch.long), persistent=True)
        self.r, self.alpha, self.scale = r, alpha, alpha / r
        self.A_gate = nn.Parameter(torch.empty(k, r, hidden))
        self.B_gate = nn.Parameter(torch.zeros(k, inter, r))
        self.A_up = nn.Parameter(torch.empty(k, r, hidden))
        self.B_up = nn.Parameter(torch.zeros(k, inter, r))
        self.A_down = nn.Parameter(torch.empty(k, r, inter))
        self.B_down = nn.Parameter(torch.zeros(k, hidden, r))
        for a in (self.A_gate, self.A_up, self.A_down):
            _init_a(a.data)

    def delta(self, j: int):
        """Dense weight deltas of slot j in fp32: (d_gate [I, H], d_up [I, H], d_down [H, I])."""
        s = self.scale
        return tuple(s * getattr(self, "B_" + n)[j].float() @ getattr(self, "A_" + n)[j].float()
                     for n in ("gate", "up", "down"))


class MLPLoRA(nn.Module):
    """LoRA for one gated MLP (the Qwen shared expert or the Gemma dense MLP)."""

    def __init__(self, hidden: int, inter: int, r: int = 16, alpha: float = 32.0):
        super().__init__()
        self.r, self.alpha, self.scale = r, alpha, alpha / r
        self.A_gate = nn.Parameter(torch.empty(r, hidden))
        self.B_gate = nn.Parameter(torch.zeros(inter, r))
        self.A_up = nn.Parameter(torch.empty(r, hidden))
        self.B_up = nn.Parameter(torch.zeros(inter, r))
        self.A_down = nn.Parameter(torch.empty(r, inter))
        self.B_down = nn.Parameter(torch.zeros(hidden, r))
        for a in (self.A_gate, self.A_up, self.A_down):
            _init_a(a.data)

    def delta(self):
        s = self.scale
        return tuple(s * getattr(self, "B_" + n).float() @ getattr(self, "A_" + n).float()
                     for n in ("gate", "up", "down"))


class LayerLoRA(nn.Module):
    def __init__(self, experts, shared):
        super().__init__()
        self.experts = experts
        self.shared = shared


class BlockLoRA(nn.Module):
    """All LoRA modules of the trained block, keyed by absolute layer index (smel/lora.py:93-125)."""

    def __init__(self, layers: dict):
        super().__init__()
        self.layers = nn.ModuleDict({str(k): v for k, v in layers.items()})

    def get(self, l: int):
        return self.layers[str(l)] if str(l) in self.layers else None

    @classmethod
    def build(cls, selection: dict, hidden: int, inter: int, shared_inter: int, r: int, alpha: float,
              shared: bool = True):
        """selection: {layer: [expert ids]}"""
        layers = {}
        for l, ids in selection.items():
            ex = ExpertsLoRA(ids, hidden, inter, r, alpha) if len(ids) else None
            sh = MLPLoRA(hidden, shared_inter, r, alpha) if shared else None
            layers[int(l)] = LayerLoRA(ex, sh)
        return cls(layers)

    @classmethod
    def load(cls, path, dims, device="cuda"):
        """Adapter folder (adapter_config.json + adapter.safetensors, keys layers.{l}.experts.* / .shared.*)
        -> (BlockLoRA, meta)."""
        from safetensors.torch import load_file
        with open(os.path.join(path, "adapter_config.json")) as f:
            meta = json.load(f)
        experts = {int(k): v for k, v in meta["experts"].items()}
        lora = cls.build(experts, dims.hidden, dims.moe_inter, dims.shared_inter, meta["r"], meta["alpha"],
                         shared=meta["shared_lora"])
        lora.load_state_dict(load_file(os.path.join(path, "adapter.safetensors")))
        return lora.to(device), meta
