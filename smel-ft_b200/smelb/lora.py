"""LoRA parameters of the selected routed experts and of the shared expert / dense MLP (smel/lora.py:1-125).

Parameter names, shapes and initialisation follow the reference so adapters load unchanged:
  ExpertsLoRA (k slots): A_gate/A_up [k, r, H], B_gate/B_up [k, I, r], A_down [k, r, I], B_down [k, H, r]
  MLPLoRA:               A_gate/A_up [r, H],    B_gate/B_up [I, r],    A_down [r, I],    B_down [H, r]
A is initialised like PEFT (kaiming_uniform_(a=sqrt(5)) per [r, in] matrix), B with zeros, scale = alpha / r.

lora_linear / lora_gate_up (smel/lora.py:61-83) run on the GEMM engine: the LoRA term is one more 64-wide k-block
of the base GEMM's accumulation (smelb_lora_linear_fwd / _bwd), differentiable w.r.t. x, A and B.
"""
import json
import math
import os

import torch
from torch import nn

from . import _lib


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


class _LoraLinearFn(torch.autograd.Function):
    """y = x w^T + s (x A^T) B^T over 2-D bf16 x, with zero, one or two (A, B) pairs (see smelb_lora_linear_fwd).
    Gradients: x, and every A / B that requires one; the base weight w is frozen (as in the reference's use)."""

    @staticmethod
    def forward(ctx, x, w, scale, A0, B0, A1, B1):
        if w.requires_grad:
            raise _lib.SmelbError("lora_linear: the base weight is frozen here (no gradient for w)")
        T, Kd = x.shape
        N = w.shape[0]
        has_lora = A0 is not None
        r = A0.shape[0] if has_lora else 0
        npairs = 0 if not has_lora else (2 if A1 is not None else 1)
        a32 = [None if p is None else p.detach().float().contiguous() for p in (A0, B0, A1, B1)]
        dev = x.device
        y = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
        xa = torch.empty(T, 64, dtype=torch.bfloat16, device=dev) if has_lora else None
        nb = int(_lib.load().smelb_lora_linear_workspace_bytes(T, Kd, N))
        ws = torch.empty(max(nb, 256), dtype=torch.uint8, device=dev)
        _lib.call("smelb_lora_linear_fwd", _lib.ptr(x), T, Kd, _lib.ptr(w), N, *[_lib.ptr(p) for p in a32], r,
                  float(scale), _lib.ptr(y), _lib.ptr(xa), _lib.ptr(ws), ws.numel(), _lib.stream_ptr(dev))
        ctx.save_for_backward(x, w, xa, *a32)
        ctx.meta = (float(scale), r, npairs, [None if p is None else p.dtype for p in (A0, B0, A1, B1)])
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, xa, *a32 = ctx.saved_tensors
        scale, r, npairs, dtypes = ctx.meta
        T, Kd = x.shape
        N = w.shape[0]
        dev = x.device
        dy = dy.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(x) if ctx.needs_input_grad[0] else None
        grads = [None] * 4
        for i in range(2 * npairs):
            if ctx.needs_input_grad[3 + i]:
                grads[i] = torch.empty(a32[i].shape, dtype=torch.float32, device=dev)
        nb = int(_lib.load().smelb_lora_linear_workspace_bytes(T, Kd, N))
        ws = torch.empty(max(nb, 256), dtype=torch.uint8, device=dev)
        _lib.call("smelb_lora_linear_bwd", _lib.ptr(x), _lib.ptr(dy), T, Kd, _lib.ptr(w), N,
                  *[_lib.ptr(p) for p in a32], r, scale, _lib.ptr(xa), _lib.ptr(dx), _lib.ptr(grads[0]),
                  _lib.ptr(grads[1]), _lib.ptr(grads[2]), _lib.ptr(grads[3]), _lib.ptr(ws), ws.numel(),
                  _lib.stream_ptr(dev))
        grads = [None if g is None else g.to(dt) for g, dt in zip(grads, dtypes)]
        return (dx, None, None, *grads)


def _rows(x, what):
    if not x.is_cuda:
        raise _lib.SmelbError(f"{what}: smelb runs on CUDA tensors only")
    if x.dtype != torch.bfloat16:
        raise _lib.SmelbError(f"{what}: expected bf16 activations, got {x.dtype}")
    return x.reshape(-1, x.shape[-1]).contiguous()


def lora_linear(x, w, A, B, scale):
    """x @ w.T + scale * (x @ A.T) @ B.T (smel/lora.py:61-69), the LoRA term added inside the base GEMM's fp32
    accumulation before the one rounding. x [..., in] bf16, w [out, in] bf16 (frozen), A [r, in] / B [out, r]
    (fp32 parameters, or None for the plain projection)."""
    x2 = _rows(x, "lora_linear")
    w = w.to(torch.bfloat16).contiguous()
    y = _LoraLinearFn.apply(x2, w, scale, A, B, None, None)
    return y.reshape(*x.shape[:-1], w.shape[0])


def lora_gate_up(x, w_gate_up, A_gate, B_gate, A_up, B_up, scale):
    """(gate, up) of a gated MLP over the stacked weight [2I, H] (smel/lora.py:72-83): one GEMM for both halves, the
    two LoRA pairs as one 64-wide k-block ([x A_gate^T | x A_up^T] against a block-diagonal [s B_gate, s B_up])."""
    x2 = _rows(x, "lora_gate_up")
    w = w_gate_up.to(torch.bfloat16).contiguous()
    I = w.shape[0] // 2
    if A_gate is None:
        y = _LoraLinearFn.apply(x2, w, scale, None, None, None, None)
    else:
        y = _LoraLinearFn.apply(x2, w, scale, A_gate, B_gate, A_up, B_up)
    return y[:, :I], y[:, I:]


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
