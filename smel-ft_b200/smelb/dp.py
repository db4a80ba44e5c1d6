"""Data parallelism for the MoE layer: every rank holds the whole layer and runs it on its own tokens; the trainable
LoRA gradients are summed over the ranks once per step.

On a B200 the int4 banks of a layer (0.4-0.5 GB at the Qwen3.6 shape) are a small part of the 180 GB of HBM, so
replicating the layer costs little and the only exchange of a step is this all-reduce (about 1.5 MB of fp32 gradients
for the config-2 layer). Expert parallelism (`smelb.ep`) is the alternative when the banks do not fit one GPU.
"""
import torch
import torch.distributed as dist


class GradAllReduce:
    """Sums the gradients of `params` over the ranks of `group` with one all-reduce of their concatenation.

    The flat buffer is allocated once (on the first call, from the first gradient's device) and reused; parameters
    without a gradient are skipped, so the set of gradients must be the same on every rank."""

    def __init__(self, params, group=None):
        self.params = list(params)
        self.group = group
        self.buf = None

    def __call__(self):
        grads = [p.grad for p in self.params if p.grad is not None]
        if not grads:
            return
        n = sum(g.numel() for g in grads)
        if self.buf is None or self.buf.numel() != n or self.buf.device != grads[0].device:
            self.buf = torch.empty(n, dtype=torch.float32, device=grads[0].device)
        torch.cat([g.reshape(-1).float() for g in grads], out=self.buf)
        dist.all_reduce(self.buf, group=self.group)
        o = 0
        for g in grads:
            g.view(-1).copy_(self.buf[o:o + g.numel()].view_as(g.view(-1)))
            o += g.numel()


def allreduce_lora_grads(lora_layer, group=None):
    """One-off form of GradAllReduce over every parameter of `lora_layer` (a smelb.LayerLoRA or any module)."""
    if lora_layer is None:
        return
    GradAllReduce(lora_layer.parameters(), group)()
