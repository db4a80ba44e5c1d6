"""Layer-major training over a stack of MoE layers (smel/layer_runner.py:295-371, LayerMajorRunner).

Forward: every layer is taken from the source once and applied to all micro-batches under no_grad, each layer's inputs
checkpointed. Backward: the layers are taken again in reverse order; every micro-batch is recomputed under autograd
from its checkpoint and back-propagated with the gradient arriving from the layer above, which accumulates the LoRA
gradients and yields the gradient of the layer's input. The layer function defaults to the MoE block of a decoder
layer after its attention part, h + moe_forward(h) (the reference's layer_forward adds moe_forward to the residual
stream the same way; attention, norms and the LM head are outside this library's path), so the runner drives exactly
the unit smelb accelerates. Expert-parallel stacks pass `layer_fn=ep_layer_fn(comm, top_k)` and layers that are
(W, EPShard) pairs.
"""
import torch

from .moe import moe_forward


def moe_block(top_k):
    """layer_fn of the MoE block: layer = (W, LayerExperts), h + moe_forward(h, W, experts, top_k, lora)."""
    def fn(h, layer, lora, stats=None):
        W, ex = layer
        return h + moe_forward(h, W, ex, top_k, lora, stats)
    return fn


def ep_layer_fn(comm, top_k, cap_factor=2.0):
    """layer_fn of the expert-parallel MoE block: layer = (W, EPShard), the shard's LoRA (its selected experts and
    the replicated shared LoRA) is used; `lora` is ignored."""
    from .ep import moe_forward_ep

    def fn(h, layer, lora, stats=None):
        W, shard = layer
        return h + moe_forward_ep(h, W, shard, top_k, comm, stats, cap_factor)
    return fn


class _ListSource:
    def __init__(self, layers):
        self.layers = layers

    def get(self, l):
        return self.layers[l]

    def prefetch(self, l):
        pass


class LayerMajorRunner:
    """Runs layers `layers` (ids in bottom-up order) on a list of micro-batches, layer by layer.

    source: an object with get(l) / prefetch(l) (smelb.stream.LayerSource, DictSource) or a dict / list of layers;
    lora: an object with get(l) -> LayerLoRA or None (smelb.BlockLoRA) or None; layer_fn(h, layer, lora, stats) -> h';
    ckpt_device: where the forward keeps its checkpoints (None: where they are)."""

    def __init__(self, source, layers, lora=None, layer_fn=None, top_k=8, ckpt_device=None):
        self.src = source if hasattr(source, "get") and hasattr(source, "prefetch") else _ListSource(source)
        self.layers = list(layers)
        self.lora = lora
        self.layer_fn = layer_fn or moe_block(top_k)
        self.ckpt_device = ckpt_device

    def _lora(self, l):
        return self.lora.get(l) if self.lora is not None else None

    def _get(self, i, order):
        layer = self.src.get(order[i])
        if i + 1 < len(order):
            self.src.prefetch(order[i + 1])
        return layer

    @torch.no_grad()
    def forward(self, hs, keep_ckpt=False, stats_cb=None):
        """hs: list of [T_m, H] hidden states (replaced in place by the top layer's outputs). Returns (hs, ckpt)
        with ckpt[l] the inputs of layer l when keep_ckpt."""
        ckpt = {}
        order = self.layers
        for i, l in enumerate(order):
            layer = self._get(i, order)
            if keep_ckpt:
                ckpt[l] = [h if self.ckpt_device is None else h.to(self.ckpt_device, non_blocking=True) for h in hs]
            for m in range(len(hs)):
                st = (lambda p, v, t, _l=l, _m=m: stats_cb(_l, _m, p, v, t)) if stats_cb else None
                hs[m] = self.layer_fn(hs[m], layer, self._lora(l), st)
        return hs, ckpt

    def backward(self, ckpt, grads):
        """grads: the loss gradients w.r.t. the top layer's outputs, one per micro-batch; returns the gradients
        w.r.t. the bottom layer's inputs. The LoRA gradients accumulate in their parameters."""
        order = self.layers[::-1]
        for i, l in enumerate(order):
            layer = self._get(i, order)
            for m in range(len(grads)):
                x = ckpt[l][m].to(grads[m].device, non_blocking=True).detach().requires_grad_(True)
                with torch.enable_grad():
                    y = self.layer_fn(x, layer, self._lora(l))
                    y.backward(grads[m])
                grads[m] = x.grad
                ckpt[l][m] = None
        return grads

    def train_step(self, hs, grad_fn):
        """forward with checkpoints, grads = grad_fn(top outputs) (the loss head's gradients, e.g. from
        smelb.chunked_ce), backward. Returns (grads w.r.t. the bottom inputs, grad_fn's other outputs)."""
        hs, ckpt = self.forward(hs, keep_ckpt=True)
        grads, extra = grad_fn(hs)
        del hs
        return self.backward(ckpt, list(grads)), extra
