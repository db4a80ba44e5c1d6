"""Layer weight sources for layer-major training (smel/stream.py:16-114): the layer's tensors live in pinned host
memory and are copied to the GPU while the previous layer computes.

B200 design: the copies are asynchronous host-to-device copies from pinned memory on a dedicated copy stream (the
host never blocks, so no worker thread is needed as in the reference, whose thread also reads mmap'd files); the
consumer stream waits on an event recorded after the copies, and every uploaded tensor is `record_stream`ed on the
consumer so the caching allocator cannot hand its memory out again while a kernel of that layer may still read it.
With `resident=True` (the right choice on a 180 GB B200 whenever the banks fit: about 0.45 GB of int4 experts per
Qwen3.6 layer, 17 GB for 40 layers) every layer is uploaded once and kept.

Layer dicts use the reference's packed keys (smel/stream.py:16-36, smel/pack.py:8-25):
  experts.gate_up.{q,scale,zero}, experts.down.{q,scale,zero}   the int4 bank
  experts.sel.gate_up, experts.sel.down, experts.sel.ids         the bf16 copies of the selected experts
  mlp.experts.gate_up_proj, mlp.experts.down_proj                a bf16 bank instead of the int4 one
  everything else                                                dense tensors (router, shared expert, norms)
"""
import torch

from .moe import BF16Experts, Int4Experts, LayerExperts


def build_layer(t: dict, sel_ids=None, group: int = 32, frozen_dtype=torch.bfloat16, act: str = "silu"):
    """(dense, LayerExperts) from one layer's device tensors (names relative to the layer), as
    smel/stream.py:16-36 build_layer: a bf16 fused bank ('mlp.experts.*') or the packed int4 bank ('experts.*')
    plus the selected experts' bf16 copies ('experts.sel.*')."""
    dense = {k: v for k, v in t.items() if not k.startswith(("mlp.experts.", "experts."))}
    if "mlp.experts.gate_up_proj" in t:
        gu, dn = t["mlp.experts.gate_up_proj"], t["mlp.experts.down_proj"]
        frozen = BF16Experts(gu, dn)
        sgu = sdn = None
        if sel_ids is not None and len(sel_ids):
            ids = torch.as_tensor(sel_ids, device=gu.device)
            sgu, sdn = gu[ids].clone(), dn[ids].clone()
    else:
        gq = {k[len("experts.gate_up."):]: v for k, v in t.items() if k.startswith("experts.gate_up.")}
        dq = {k[len("experts.down."):]: v for k, v in t.items() if k.startswith("experts.down.")}
        frozen = Int4Experts(gq, dq, dtype=frozen_dtype)
        sgu, sdn = t.get("experts.sel.gate_up"), t.get("experts.sel.down")
        if sel_ids is None and "experts.sel.ids" in t:
            sel_ids = t["experts.sel.ids"].tolist()
    if sgu is None:
        sel_ids = None
    return dense, LayerExperts(frozen, sel_ids, sgu, sdn, group=group, act=act)


class LayerSource:
    """Layers from host dicts {l: {name: CPU tensor}} with double-buffered upload (smel/stream.py:39-114).

    get(l) returns make(l, gpu_tensors) (by default build_layer's (dense, LayerExperts)) once layer l is on the GPU;
    prefetch(l) starts its upload without waiting. At most `max_on_gpu` layers are kept unless `resident`.
    stats: bytes and loads uploaded, and `wait_ms`, the time the consumer stream spent waiting for copies (measured
    with CUDA events when `timing` is set)."""

    def __init__(self, layers: dict, device="cuda", resident=False, max_on_gpu=2, pin=True, make=None,
                 group=32, act="silu", timing=False):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("LayerSource: smelb layers run on CUDA devices")
        self.resident, self.max_on_gpu = resident, max(1, int(max_on_gpu))
        self.group, self.act, self.timing = group, act, timing
        self.make = make or (lambda l, t: build_layer(t, None, self.group, act=self.act))
        self.host = {}
        for l, t in layers.items():
            self.host[l] = {k: (v.pin_memory() if pin and not v.is_pinned() else v) for k, v in t.items()}
        self.copy = torch.cuda.Stream(self.device)
        self.cache = {}    # l -> built layer (most recently used last)
        self.pending = {}  # l -> (gpu tensors, copy-done event)
        self.stats = {"bytes": 0, "loads": 0, "wait_ms": 0.0}
        self._waits = []
        if resident:
            for l in self.host:
                self.prefetch(l)

    def _evict(self, keep):
        if self.resident:
            return
        while len(self.cache) + len(self.pending) > self.max_on_gpu:
            victims = [k for k in self.cache if k != keep]
            if not victims:
                break
            del self.cache[victims[0]]

    def prefetch(self, l):
        """Start copying layer l to the GPU on the copy stream (no host wait)."""
        if l in self.cache or l in self.pending:
            return
        if not self.resident:
            while len(self.cache) + len(self.pending) >= self.max_on_gpu and self.cache:
                del self.cache[next(iter(self.cache))]
        # New allocations on the copy stream: an evicted layer's memory is not reused before the consumer's work on
        # it finished, because get() record_stream'ed every tensor on the consumer stream.
        with torch.cuda.stream(self.copy):
            gpu = {k: v.to(self.device, non_blocking=True) for k, v in self.host[l].items()}
            done = torch.cuda.Event(enable_timing=self.timing)
            done.record(self.copy)
        self.stats["bytes"] += sum(v.numel() * v.element_size() for v in gpu.values())
        self.stats["loads"] += 1
        self.pending[l] = (gpu, done)

    def get(self, l):
        """Layer l, uploaded and built; the current stream waits for its copies."""
        if l in self.cache:
            layer = self.cache.pop(l)
            self.cache[l] = layer
            return layer
        if l not in self.pending:
            self.prefetch(l)
        gpu, done = self.pending.pop(l)
        cur = torch.cuda.current_stream(self.device)
        if self.timing:
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(cur)
            self._waits.append((t0, done))
        cur.wait_event(done)
        for v in gpu.values():
            v.record_stream(cur)
        layer = self.make(l, gpu)
        self.cache[l] = layer
        self._evict(keep=l)
        return layer

    def wait_ms(self):
        """Consumer-stream time spent waiting for uploads so far (needs timing=True and a synchronised device)."""
        for t0, done in self._waits:
            self.stats["wait_ms"] += max(0.0, t0.elapsed_time(done))
        self._waits.clear()
        return self.stats["wait_ms"]

    def close(self):
        torch.cuda.current_stream(self.device).wait_stream(self.copy)
        self.cache.clear()
        self.pending.clear()


class DictSource:
    """Already materialised layers (smel/stream.py:200-214): get returns them as they are."""

    def __init__(self, layers: dict):
        self.layers = layers
        self.stats = {"bytes": 0, "loads": 0, "wait_ms": 0.0}

    def get(self, l):
        return self.layers[l]

    def prefetch(self, l):
        pass

    def close(self):
        pass
