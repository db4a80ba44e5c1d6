"""Benchmark of the SMEL FT MoE expert layer on B200: tokens/s of forward + recompute + backward at the
Qwen3.6-35B-A3B layer shape (config 2), as one JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = the layer-major training unit of the reference (smel/layer_runner.py:319-364): a no-grad forward of the
micro-batch, then a recompute under autograd and the backward (dX plus all LoRA gradients), on 4092 tokens of seeded
synthetic input (Zipf-skewed routing, 244 int4 + 12 bf16 LoRA experts, shared expert with LoRA).
With N > 1 (torchrun) every rank brings its own 4092 tokens (weak scaling) and the step time is the maximum over
ranks: by default (`--parallel dp`) every GPU holds the whole layer and the LoRA gradients are all-reduced every step;
`--parallel ep` splits the experts over the GPUs instead (smelb.ep, row all-to-alls over NCCL).
`--impl reference` times the CPU restatement of the reference's torch path on the host cores instead.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "smel-ft_b200"))
sys.path.insert(0, ROOT)

METRIC = "MoE-layer tokens/s fwd+recompute+bwd (Qwen3.6 shape) and % of HBM/TC roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.path, self.skip = index, None, None, 0

    def start(self, settle_s=10.0):
        """Start sampling and return once the first sample is written, so that nvidia-smi's start-up (NVML
        initialisation) is over before the timed region begins."""
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.index)], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < settle_s and os.path.getsize(self.path) == 0:
            time.sleep(0.05)
        self.skip = sum(1 for _ in open(self.path))  # samples taken before the timed region

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for i, line in enumerate(open(self.path)):
            if i < self.skip:
                continue
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "window": "1 s of warm-up replays of the same step, then the timed region"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def steps_for(seconds, t0, done, world):
    """The number of further steps that fill `seconds`, from `done` steps timed since perf_counter() t0 (after a
    synchronize) and agreed by every rank (the slowest one's step time): each step holds collectives, so every rank
    must take the same number of them."""
    per = max_over_ranks((time.perf_counter() - t0) / max(done, 1), world)
    return max(1, int(math.ceil(seconds / max(per, 1e-6))))


def layer_config(args):
    return dict(T=args.tokens, H=2048, E=256, K=8, I=512, S=512, n_sel=12, r=16, alpha=32.0)


def config_json(cfg, meta, world, parallel="dp"):
    return {"workload": "qwen3.6-35b-a3b moe layer (config 2): fwd + recompute + bwd", "tokens": cfg["T"],
            "hidden": cfg["H"], "experts": cfg["E"], "top_k": cfg["K"], "expert_inter": cfg["I"],
            "shared_inter": cfg["S"], "frozen": "int4 group-64", "lora_experts": cfg["n_sel"],
            "lora_rank": cfg["r"], "routing": "zipf s=1.1 over a seeded permutation, temperature bisected so the "
            "12 LoRA experts hold 50% +- 2% of the renormalised top-8 gate mass", "seed": meta.get("seed"),
            "l2": "weights 0.53 GB > L2 126 MB: each step streams the banks from HBM",
            "parallelism": "single" if world == 1 else
            (f"ep{world}: experts split over {world} GPUs (load-balanced placement), rows exchanged over NVLink through "
             f"peer memory, {cfg['T']} tokens per GPU (weak scaling)" if parallel == "ep"
             else f"dp{world}: the whole layer on each of {world} GPUs, {cfg['T']} tokens per GPU (weak scaling), "
                  f"LoRA gradients all-reduced every step")}


# ------------------------------------------------------------------------------------------ CPU baseline
def cpu_model():
    """The host CPU's model name (lscpu's "Model name", read from /proc/cpuinfo)."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _time_cpu_step(p, tokens, dtype):
    from oracle import cpu_step
    gy = torch.randn(p["x"].shape, generator=torch.Generator().manual_seed(9)).to(dtype)
    small = dict(p)
    small["x"] = p["x"][:64]
    cpu_step.step(small, gy[:64])  # warm-up (allocator, thread pool)
    t0 = time.perf_counter()
    cpu_step.step(p, gy)
    return time.perf_counter() - t0


def cpu_baseline(layer, tokens, bf16_tokens=1024):
    """The reference's torch CPU path (oracle/cpu_step.py) on the host cores: `tokens` tokens in fp32 (the headline
    value) and `bf16_tokens` in bf16, one warm-up + one timed step each."""
    from oracle import cpu_step
    torch.set_num_threads(os.cpu_count() or 1)
    dt = _time_cpu_step(cpu_step.prepare(layer, dtype=torch.float32, tokens=tokens), tokens, torch.float32)
    res = {"value": tokens / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
           "cpu_model": cpu_model(),
           "sample": f"{tokens} tokens of the same layer, 1 step (fwd no-grad + recompute + bwd), float32, {dt:.2f} s"}
    if bf16_tokens:
        db = _time_cpu_step(cpu_step.prepare(layer, dtype=torch.bfloat16, tokens=bf16_tokens), bf16_tokens,
                            torch.bfloat16)
        res["bf16"] = {"value": bf16_tokens / db, "unit": "tokens/s",
                       "sample": f"{bf16_tokens} tokens of the same layer, 1 step, bfloat16, {db:.2f} s"}
    return res


# ------------------------------------------------------------------------------------------ our arm
def run_ours(args, world, rank, local):
    import smelb
    from smelb import _lib
    from smelb.synth import flops_per_token, qwen_layer
    dev = torch.device("cuda", local)
    cfg = layer_config(args)
    ep_mode = world > 1 and args.parallel == "ep"
    dp_mode = world > 1 and args.parallel == "dp"
    # With several GPUs every rank brings its own cfg["T"] tokens (weak scaling) of one layer (same weights on every
    # rank, built from one seed). ep (default): the experts are split over the ranks with a load-balanced placement
    # (smelb.ep: rows exchanged over NVLink through peer memory, device-side synchronisation) and the replicated
    # shared expert's LoRA gradients are summed every step; dp: every GPU holds the whole layer and all LoRA gradients
    # are summed (one NCCL all-reduce of the flattened gradients).
    layer = qwen_layer(T=cfg["T"] * world, H=cfg["H"], E=cfg["E"], K=cfg["K"], I=cfg["I"], S=cfg["S"],
                       n_sel=cfg["n_sel"], r=cfg["r"], alpha=cfg["alpha"], seed=0, device=dev)
    W, ex, lora, K = layer["W"], layer["ex"], layer["lora"], cfg["K"]
    x = layer["x"][rank * cfg["T"]:(rank + 1) * cfg["T"]].contiguous()
    gy = torch.randn(x.shape, generator=torch.Generator(device=dev).manual_seed(9 + rank), device=dev).bfloat16()
    comm = shard = None
    placement_note = None
    if ep_mode:
        from smelb import ep
        rec = {}
        with torch.no_grad():  # routing of all ranks' tokens: the per-expert loads the placement balances
            smelb.moe_forward(layer["x"], W, ex, K, None, stats=lambda p, v, i: rec.update(i=i))
        loads = torch.bincount(rec["i"].reshape(-1), minlength=cfg["E"]).tolist()
        costs = ep.expert_costs(ex, loads)
        placement = ep.balanced_placement(loads, world, costs)
        per_rank = [sum(loads[e] for e in ids) for ids in placement]
        placement_note = {"placement": f"balanced by routed cost (rows, + {ep.FROZEN_TILE_COST:g} per frozen expert "
                                       f"token tile)",
                          "rows_per_rank": per_rank,
                          "cost_per_rank": [round(sum(costs[e] for e in ids)) for ids in placement]}
        shard = ep.shard_layer(ex, lora, rank, world, placement)
        comm = ep.EPGroup(cap=cfg["T"], H=cfg["H"], K=K)
        params = list(shard.lora.parameters())
        sync_params = list(shard.lora.shared.parameters())  # the replicated shared LoRA
    else:
        params = list(lora.parameters())
        sync_params = params if dp_mode else []

    def layer_call(xd):
        if ep_mode:
            return ep.moe_forward_ep(xd, W, shard, K, comm)
        return smelb.moe_forward(xd, W, ex, K, lora)

    def step(xd, gd):
        for p in params:
            p.grad = None
        with torch.no_grad():
            layer_call(xd)
        xr = xd.detach().requires_grad_(True)
        out = layer_call(xr)
        out.backward(gd)
        return xr.grad

    grad_sum = None
    if sync_params:
        from smelb import dp
        grad_sum = dp.GradAllReduce(sync_params)

    def dp_sync():
        """Sum the replicated LoRA gradients over the ranks (one all-reduce of their concatenation): all of them with
        data parallelism, the shared expert's with expert parallelism."""
        if grad_sum is not None:
            grad_sum()

    # everything runs on one side stream: a CUDA graph is captured on it, and autograd's gradient accumulation
    # nodes must live on the stream they are replayed on
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    torch.cuda.set_stream(side)
    for _ in range(args.warmup):
        step(x, gy)
        dp_sync()
    torch.cuda.synchronize()
    assert smelb.read_status() == 0, "device status word set during warm-up"

    # ---------------- end to end through the public API with host buffers
    xh = x.cpu().pin_memory()
    gh = gy.cpu().pin_memory()
    dxh = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(x) for _ in range(2)]
    gd = [torch.empty_like(gy) for _ in range(2)]
    # Every step copies its inputs from pinned host memory and reads its dX back. The copies run on their own
    # stream, double-buffered as an input pipeline would: step i+1's inputs upload while step i computes, and step
    # i's dX downloads while step i+1 computes. Measured first, before the graph capture and the clock sampler: the
    # loop drives Python, autograd and the launches every step, so nothing else may compete for the host.
    copy_s = torch.cuda.Stream(dev)
    up_done = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]   # step finished with buffer b (inputs consumed, dX produced)
    down_done = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        b = i % 2
        with torch.cuda.stream(copy_s):
            if i >= 2:
                copy_s.wait_event(used[b])
            xd[b].copy_(xh, non_blocking=True)
            gd[b].copy_(gh, non_blocking=True)
            up_done[b].record(copy_s)

    def e2e_loop(n):
        """n steps of the pipeline; returns the CUDA events around them (on the copy stream and the step stream)."""
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(copy_s)
        side.wait_event(e0)
        upload(0)
        dxs = [None, None]
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                upload(i + 1)
            side.wait_event(up_done[b])
            if i >= 2:
                side.wait_event(down_done[b])  # the host copy of dX two steps back has left this buffer's slot
            dxs[b] = step(xd[b], gd[b])
            dp_sync()
            used[b].record(side)
            with torch.cuda.stream(copy_s):
                copy_s.wait_event(used[b])
                dxh[b].copy_(dxs[b], non_blocking=True)
                down_done[b].record(copy_s)
        side.wait_stream(copy_s)
        e1.record(side)
        return e0, e1

    # untimed warm-up of the same pipeline first: the copy stream, the device buffers and the first pinned
    # transfers cost ~0.2 s once, which spread over the timed steps would halve the number
    e2e_loop(max(args.warmup, 2))
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = e2e_loop(args.steps)
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), world)
    e2e = {"value": world * cfg["T"] * args.steps / (ms_e2e / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": xh.numel() * 2 + gh.numel() * 2, "d2h_bytes_per_step": dxh[0].numel() * 2}
    assert smelb.read_status() == 0, "device status word set during the end-to-end loop"

    # ---------------- device-resident timing: the whole step (no-grad forward, recompute, backward) is captured once
    # in a CUDA graph and replayed, so the number is the device's and not the Python host's
    graph, timing = None, "cuda-graph replay of the whole step"
    n0 = _lib.launch_count()
    try:
        torch.cuda.synchronize()
        n0 = _lib.launch_count()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            step(x, gy)
        torch.cuda.synchronize()
    except Exception as exc:  # not capturable here: time the eager step instead and say so
        graph, timing = None, f"eager (graph capture failed: {str(exc).splitlines()[0][:120]})"
        torch.cuda.synchronize()
        n0 = _lib.launch_count()
    per_step_launches = _lib.launch_count() - n0 if graph is not None else None

    def run_step():
        if graph is not None:
            graph.replay()
        else:
            step(x, gy)
        dp_sync()

    # warm-up replays, then at least ~1 s more of them with the clock sampler running, so that the clock record
    # covers the GPU under this load right up to and through the timed region (a timed region of a few tens of ms
    # is shorter than the sampler's period)
    t_w = time.perf_counter()
    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    n_more = steps_for(1.0, t_w, args.warmup, world)
    clocks = Clocks(local)
    clocks.start()
    for _ in range(n_more):
        run_step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    n1 = _lib.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    e0.record()
    for _ in range(args.steps):
        run_step()
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    ck = clocks.stop()
    # kernels of this library launched in the timed region (a graph replay launches the captured ones again)
    launches = per_step_launches * args.steps if graph is not None else _lib.launch_count() - n1
    assert smelb.read_status() == 0, "device status word set during the timed region"
    # the expert-GEMM launches of the same steps, timed with CUDA events on their stream (separate pass)
    _lib.gemm_timing(True)
    _lib.gemm_timing_read()
    for _ in range(args.steps):
        step(x, gy)
    gemm_ms, gemm_n = _lib.gemm_timing_read()
    _lib.gemm_timing(False)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    ms_step = ms / args.steps
    value = world * cfg["T"] * args.steps / (ms / 1e3)

    # ---------------- roofline of the dominant kernel (the expert GEMM engine)
    with torch.no_grad():
        rec = {}
        smelb.moe_forward(x, W, ex, K, lora, stats=lambda p, v, i: rec.update(i=i))
    sel = torch.zeros(cfg["E"], dtype=torch.bool, device=dev)
    sel[layer["meta"]["selected"]] = True
    frac = float(sel[rec["i"]].float().mean())
    f_tok = flops_per_token(cfg["H"], cfg["E"], cfg["K"], cfg["I"], cfg["S"], n_lora_rows_frac=frac, r=cfg["r"])
    flops_step = 3 * f_tok * cfg["T"]  # forward + recompute + backward (dX), LoRA terms included per pass
    pk, pk_kind = peaks()
    gemm_ms_step = gemm_ms / args.steps
    achieved = flops_step / (gemm_ms_step / 1e3) / 1e12
    peak = pk["bf16_tflops"]
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "moe_gemm_traffic.json")
    if os.path.exists(tpath):  # DRAM bytes of the GEMM launches of one step, from the committed ncu capture
        tj = json.load(open(tpath))
        traffic = {"bytes_per_launch": round(tj["traffic_bytes_per_step"] / tj["launches_per_step"]),
                   "bytes_per_step": round(tj["traffic_bytes_per_step"]), "source": tj["source"]}
    roof = {"bound": "tensor", "kernel": "moe_gemm_kernel (all expert / router / LoRA GEMMs of the step)",
            "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "peak_kind": f"{pk_kind} bf16 burst", "traffic": traffic,
            "gemm_ms_per_step": round(gemm_ms_step, 4), "gemm_launches_per_step": gemm_n // max(args.steps, 1),
            "algorithmic_flops_per_step": flops_step,
            "layer_frac_of_roofline": round((flops_step / (ms_step / 1e3) / 1e12) / peak, 4)}
    res = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, random-init weights of the layer shape)",
           "config": config_json(cfg, layer["meta"], world, args.parallel), "timing": timing,
           "routing_share": round(layer["meta"].get("share", 0.0), 4), "roofline": roof,
           "e2e": e2e,
           "gpu_launches": int(launches), "clocks": ck}
    if placement_note:
        res["expert_parallel"] = placement_note
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(layer, min(cfg["T"], args.cpu_tokens))
    del graph
    if comm is not None:  # every peer has finished reading this rank's region before it is freed
        torch.cuda.synchronize()
        barrier(world)
        comm.close()
    return res


# ------------------------------------------------------------------------------------------ graph timing helper
def _time_graph(step, args, local, world, post=None):
    """Capture `step` (on a side stream) in a CUDA graph and time K replays after W warm-up replays with CUDA events,
    the clocks sampled over 1 s of replays and the timed region; eager if the capture fails. `post` (a collective,
    kept out of the graph) runs after every step, inside the timed region. Returns (ms per step (max over ranks),
    timing note, clocks, this library's launches in the timed region)."""
    from smelb import _lib
    dev = torch.device("cuda", local)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    torch.cuda.set_stream(side)
    for _ in range(max(args.warmup, 1)):
        step()
        if post is not None:
            post()
    torch.cuda.synchronize()
    graph, timing = None, "cuda-graph replay of the whole step"
    try:
        n0 = _lib.launch_count()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            step()
        per = _lib.launch_count() - n0
        torch.cuda.synchronize()
    except Exception as exc:
        graph, timing, per = None, f"eager (graph capture failed: {str(exc).splitlines()[0][:120]})", None
        torch.cuda.synchronize()
    one = graph.replay if graph is not None else step

    def run():
        one()
        if post is not None:
            post()
    t_w = time.perf_counter()
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    n_more = steps_for(1.0, t_w, args.warmup, world)
    clocks = Clocks(local)
    clocks.start()
    for _ in range(n_more):
        run()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    n1 = _lib.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    ck = clocks.stop()
    launches = per * args.steps if per is not None else _lib.launch_count() - n1
    ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    del graph
    return ms, timing, ck, int(launches)


# ------------------------------------------------------------------------------------------ config 3
def run_gemma(args, local):
    """Config 3: the Gemma-4-26B-A4B-like MoE block (smel/layer_runner.py:249-261; H 2816, 128 experts top-8, expert
    intermediate 704, dense GeGLU MLP 2112 with LoRA, 116 int4 + 12 bf16 LoRA experts, Zipf s=1.1) on 4096 tokens:
    no-grad forward, then recompute + backward of h and xm, graph-timed. One JSON line with the roofline of its
    algorithmic FLOPs (394.7 MFLOP per token over the three passes) and the CPU oracle on a token sample."""
    import smelb
    from smelb import _lib
    from smelb.synth import gemma_layer
    dev = torch.device("cuda", local)
    T, H, E, K, I, S = 4096, 2816, 128, 8, 704, 2112
    L = gemma_layer(T=T, seed=0, device=dev)
    W, ex, lora, meta = L["W"], L["ex"], L["lora"], L["meta"]
    h, xm = L["h"], L["xm"]
    gy = torch.randn(h.shape, generator=torch.Generator(device=dev).manual_seed(9), device=dev).bfloat16()
    params = list(lora.parameters())

    def step():
        for p in params:
            p.grad = None
        with torch.no_grad():
            smelb.moe_block_gemma4(h, xm, W, ex, K, meta["eps"], "gelu_tanh", lora)
        hr, xr = h.detach().requires_grad_(True), xm.detach().requires_grad_(True)
        smelb.moe_block_gemma4(hr, xr, W, ex, K, meta["eps"], "gelu_tanh", lora).backward(gy)

    ms, timing, ck, launches = _time_graph(step, args, local, 1)
    assert smelb.read_status() == 0
    _lib.gemm_timing(True)
    _lib.gemm_timing_read()
    step()
    gemm_ms, gemm_n = _lib.gemm_timing_read()
    _lib.gemm_timing(False)
    f_tok = 2 * K * 3 * H * I + 2 * 3 * H * S + 2 * H * E
    flops = 3 * f_tok * T
    pk, pk_kind = peaks()
    res = {"metric": "Gemma-4 MoE block tokens/s fwd+recompute+bwd (config 3) and % of TC roofline",
           "value": round(T / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "bf16",
           "data": "synthetic (seeded, random-init weights of the block shape)",
           "config": {"workload": "gemma-4-26b-a4b-like moe block (config 3): fwd + recompute + bwd", "tokens": T,
                      "hidden": H, "experts": E, "top_k": K, "expert_inter": I, "dense_inter": S,
                      "frozen": "int4 group-64", "lora_experts": 12, "lora_rank": 16,
                      "routing": "zipf s=1.1, the 12 LoRA experts hold 50% +- 2% of the gate mass"},
           "routing_share": round(meta["share"], 4), "timing": timing,
           "roofline": {"bound": "tensor", "achieved": round(flops / (ms / 1e3) / 1e12, 1), "peak": pk["bf16_tflops"],
                        "unit": "TFLOP/s", "frac": round(flops / (ms / 1e3) / 1e12 / pk["bf16_tflops"], 4),
                        "peak_kind": f"{pk_kind} bf16 burst", "algorithmic_flops_per_step": flops,
                        "gemm_ms_per_step": round(gemm_ms, 4), "gemm_launches_per_step": gemm_n,
                        "gemm_frac": round(flops / (gemm_ms / 1e3) / 1e12 / pk["bf16_tflops"], 4)},
           "gpu_launches": launches, "clocks": ck}
    if not args.no_cpu_baseline:
        res["cpu_baseline"] = _gemma_cpu_baseline(L, args.cpu_tokens)
    return res


def _gemma_cpu_baseline(L, tokens):
    """The reference's torch path of the Gemma block (restated in oracle/moe_oracle.py) on the host cores, fp32,
    forward + recompute + backward on a token sample."""
    from oracle import moe_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    tokens = min(tokens, 512)
    W = {k: v.float().cpu() for k, v in L["W"].items()}
    ex, lora, meta = L["ex"], L["lora"], L["meta"]
    q = {k: v.cpu() for k, v in ex.frozen.gu.items()}, {k: v.cpu() for k, v in ex.frozen.dn.items()}

    class Lazy:  # the reference dequantizes the frozen experts per call (smel/quant.py:87-94)
        def __init__(self, d):
            self.d, self.shape = d, (d["q"].shape[0], d["q"].shape[1], d["q"].shape[2] * 2)

        def __getitem__(self, e):
            return O.dequant_int4(self.d["q"][e], self.d["scale"][e], self.d["zero"][e])

    names = ("A_gate", "B_gate", "A_up", "B_up", "A_down", "B_down")
    s = lora.experts.scale
    lex = {n: getattr(lora.experts, n).detach().cpu().float().requires_grad_(True) for n in names}
    lsh = {n: getattr(lora.shared, n).detach().cpu().float().requires_grad_(True) for n in names}
    h, xm = L["h"][:tokens].float().cpu(), L["xm"][:tokens].float().cpu()
    sel = ex.sel_ids.tolist()

    def run(hh, xx):
        return O.moe_block_gemma4(hh, xx, W, Lazy(q[0]), Lazy(q[1]), 8, meta["eps"], sel, ex.sel_gate_up.float().cpu(),
                                  ex.sel_down.float().cpu(), {**lex, "scale": s}, {**lsh, "scale": s}, "gelu_tanh")[0]
    gy = torch.randn(h.shape, generator=torch.Generator().manual_seed(9))
    t0 = time.perf_counter()
    with torch.no_grad():
        run(h, xm)
    hr, xr = h.clone().requires_grad_(True), xm.clone().requires_grad_(True)
    run(hr, xr).backward(gy)
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{tokens} tokens of the same block, 1 step (fwd no-grad + recompute + bwd), float32, {dt:.2f} s"}


# ------------------------------------------------------------------------------------------ config 5
def run_block(args, world, rank, local, n_layers=24, n_micro=16):
    """Config 5: a layer-major block of 24 Qwen3.6-shape MoE layers (smel/layer_runner.py:295-371 with the MoE block
    h + moe(h) of every layer), 16 micro-batches of 4092 tokens per rank: forward of every layer over all micro-
    batches, then recompute + backward in reverse layer order (smelb.runner.LayerMajorRunner). With N > 1 the experts
    of every layer are split over the GPUs (expert parallel, load-balanced placement) and each rank brings its own
    16 micro-batches (weak scaling); the shared experts' LoRA gradients are summed every step. Every layer has its own
    expert bank, selected experts, LoRA and shared expert; the router of layer 0 is used by all layers so that each
    layer sees the configured Zipf skew on the residual stream. One JSON line on rank 0: whole-box tokens/s."""
    import smelb
    from smelb import ep
    from smelb.runner import LayerMajorRunner, ep_layer_fn, moe_block
    from smelb.synth import qwen_layer
    dev = torch.device("cuda", local)
    cfg = layer_config(args)
    T, K = cfg["T"], cfg["K"]
    layers, loras, comm, router, placement, x_all = {}, {}, None, None, None, None
    if world > 1:
        comm = ep.EPGroup(cap=T, H=cfg["H"], K=K)
    for l in range(n_layers):
        Ly = qwen_layer(T=(world * n_micro * T if l == 0 else 64), H=cfg["H"], E=cfg["E"], K=K, I=cfg["I"], S=cfg["S"],
                        n_sel=cfg["n_sel"], r=cfg["r"], alpha=cfg["alpha"], seed=100 + l, device=dev)
        W = Ly["W"]
        if l == 0:
            router = W["mlp.gate.weight"]
            x_all = Ly["x"]
            if world > 1:
                rec = {}
                with torch.no_grad():
                    smelb.moe_forward(x_all[:n_micro * T], W, Ly["ex"], K, None, stats=lambda p, v, i: rec.update(i=i))
                loads = torch.bincount(rec["i"].reshape(-1), minlength=cfg["E"]).tolist()
                placement = ep.balanced_placement(loads, world, ep.expert_costs(Ly["ex"], loads))
        else:
            W["mlp.gate.weight"] = router
        if world > 1:
            shard = ep.shard_layer(Ly["ex"], Ly["lora"], rank, world, placement)
            layers[l], loras[l] = (W, shard), shard.lora
        else:
            layers[l], loras[l] = (W, Ly["ex"]), Ly["lora"]
        del Ly
        torch.cuda.empty_cache()
    xs = [x_all[(rank * n_micro + m) * T:(rank * n_micro + m + 1) * T].contiguous() for m in range(n_micro)]
    del x_all
    g = torch.Generator(device=dev).manual_seed(9 + rank)
    gys = [torch.randn(x.shape, generator=g, device=dev).bfloat16() for x in xs]
    block = smelb.BlockLoRA(loras)
    params = list(block.parameters())
    shared = [p for lo in loras.values() for p in lo.shared.parameters()]
    runner = LayerMajorRunner(layers, range(n_layers), lora=block,
                              layer_fn=ep_layer_fn(comm, K) if world > 1 else moe_block(K))
    from smelb import dp
    sync = dp.GradAllReduce(shared) if world > 1 else None

    def step():
        for p in params:
            p.grad = None
        runner.train_step([x.clone() for x in xs], lambda hs: ([gy.clone() for gy in gys], None))

    ms_total, timing, ck, launches = _time_graph(step, args, local, world, post=sync)
    assert smelb.read_status() == 0
    toks = world * n_micro * T
    res = {"metric": "layer-major block tokens/s (24 Qwen3.6-shape MoE layers, 16 micro-batches, config 5)",
           "value": round(toks / (ms_total / 1e3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms_total, 3), "higher_is_better": True, "scaling": "weak",
           "dtype": "bf16", "data": "synthetic (seeded, random-init weights of the layer shape)",
           "config": {"workload": "config 5: 24-layer MoE block, forward of all micro-batches then recompute + bwd",
                      "layers": n_layers, "micro_batches": n_micro, "tokens_per_micro_batch": T,
                      "parallelism": "single" if world == 1 else
                      f"ep{world}: experts of every layer split over {world} GPUs (load-balanced), "
                      f"{n_micro} micro-batches of {T} tokens per GPU (weak scaling)"},
           "timing": timing + ("; the shared-LoRA gradient all-reduce after every replay, in the timed region"
                               if world > 1 else ""),
           "gpu_launches": launches, "clocks": ck}
    torch.cuda.synchronize()
    barrier(world)
    if comm is not None:
        comm.close()
    return res


# ------------------------------------------------------------------------------------------ layer streaming
def run_stream(args, local, n_layers=4):
    """Layer-major forward over a stack of config-2 layers (smel/layer_runner.py:319-330 with stream.py:90-110): each
    layer's packed tensors come from pinned host memory through smelb.stream.LayerSource (two layers on the GPU,
    the next one uploading while the current one computes), against the same stack kept resident. One JSON line per
    mode: tokens/s of one pass over the stack, the bytes uploaded per pass and the time the compute stream waited."""
    import smelb
    from smelb.stream import LayerSource
    from smelb.synth import qwen_layer
    dev = torch.device("cuda", local)
    cfg = layer_config(args)
    host, x = {}, None
    for l in range(n_layers):
        L = qwen_layer(T=cfg["T"], H=cfg["H"], E=cfg["E"], K=cfg["K"], I=cfg["I"], S=cfg["S"], n_sel=cfg["n_sel"],
                       r=cfg["r"], alpha=cfg["alpha"], seed=20 + l, device=dev, with_lora=False)
        ex = L["ex"]
        t = dict(L["W"])
        t.update({"experts.gate_up." + k: v for k, v in ex.frozen.gu.items()})
        t.update({"experts.down." + k: v for k, v in ex.frozen.dn.items()})
        t.update({"experts.sel.gate_up": ex.sel_gate_up, "experts.sel.down": ex.sel_down,
                  "experts.sel.ids": ex.sel_ids.clone()})
        host[l] = {k: v.cpu() for k, v in t.items()}
        x = L["x"] if x is None else x
        del L, ex, t
    torch.cuda.empty_cache()
    for mode in ("streamed", "resident"):
        src = LayerSource(host, device=dev, resident=(mode == "resident"), max_on_gpu=2, timing=True)

        def one_pass():
            h = x
            for l in range(n_layers):
                dense, ex = src.get(l)
                src.prefetch((l + 1) % n_layers)
                h = smelb.moe_forward(h, dense, ex, cfg["K"], None)
            return h

        with torch.no_grad():
            for _ in range(2):
                one_pass()
            torch.cuda.synchronize()
            src.wait_ms()
            src.stats.update(bytes=0, loads=0, wait_ms=0.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                one_pass()
            e1.record()
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        line = {"stream": f"layer-major forward over {n_layers} config-2 layers", "mode": mode,
                "layers": n_layers, "tokens": cfg["T"], "ms_per_pass": round(ms, 3),
                "tokens_per_s_per_layer": round(cfg["T"] * n_layers / (ms / 1e3), 1),
                "h2d_gb_per_pass": round(src.stats["bytes"] / args.steps / 1e9, 3),
                "h2d_gbs": round(src.stats["bytes"] / args.steps / (ms / 1e3) / 1e9, 1),
                "compute_wait_ms_per_pass": round(src.wait_ms() / args.steps, 3)}
        print(json.dumps(line), flush=True)
        src.close()
        del src
        torch.cuda.empty_cache()


# ------------------------------------------------------------------------------------------ chunked CE
def run_ce(args, local):
    """The step after the layer stack in training (smel/loss.py chunked_ce): cross-entropy loss and dL/dh over a
    frozen LM head of the Qwen3.6 shape (hidden 2048, vocabulary 248320) on 4092 supervised rows, bf16 and int8
    heads, at the reference's default chunking (vocabulary 32768, tokens 1024) and with all rows in one token chunk.
    One JSON line per case: rows/s, the two GEMMs' share, and TFLOP/s of the 4 N V H algorithmic FLOPs against the
    measured bf16 peak; the CPU oracle on a bounded sample of rows for scale."""
    import smelb
    from smelb import _lib
    dev = torch.device("cuda", local)
    N, H, V = args.tokens, 2048, 248320
    g = torch.Generator(device=dev).manual_seed(11)
    W = (torch.randn(V, H, device=dev, generator=g) * 0.02).bfloat16()
    h = torch.randn(N, H, device=dev, generator=g).bfloat16().requires_grad_(True)
    tgt = torch.randint(0, V, (N,), device=dev, generator=g)
    pk, src = peaks()
    flops = 4.0 * N * V * H
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import ce_oracle
        torch.set_num_threads(os.cpu_count() or 1)
        rows = min(N, 1024)
        hc, tc_, wc = h.detach()[:rows].cpu(), tgt[:rows].cpu(), W.cpu()
        t0 = time.perf_counter()
        ce_oracle.chunked_ce(hc, tc_, float(rows), w=wc, vocab_chunk=32768, token_chunk=1024)
        dt = time.perf_counter() - t0
        cpu = {"value": round(rows / dt, 2), "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{rows} rows of the same head (bf16, chunks 32768 x 1024), loss + gradient, {dt:.2f} s"}
    for int8 in (False, True):
        head = smelb.LMHead.from_weight(W, int8=int8, vocab_chunk=32768)
        for tc in (1024, N):
            def step():
                h.grad = None
                smelb.chunked_ce(h, head, tgt, float(N), tc).backward()
            for _ in range(max(3, args.warmup)):
                step()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n0 = _lib.launch_count()
            torch.cuda.nvtx.range_push(f"timed_ce_{'int8' if int8 else 'bf16'}_{tc}")
            e0.record()
            for _ in range(args.steps):
                step()
            e1.record()
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            launches = (_lib.launch_count() - n0) / args.steps
            _lib.gemm_timing(True)
            step()
            gms, gn = _lib.gemm_timing_read()
            _lib.gemm_timing(False)
            tf = flops / (ms / 1e3) / 1e12
            line = {"metric": "chunked CE loss + dL/dh rows/s (Qwen3.6 LM head)", "value": round(N / (ms / 1e3), 1),
                    "unit": "rows/s", "ms_per_step": round(ms, 3), "steps": args.steps, "dtype": "bf16",
                    "data": "synthetic", "higher_is_better": True,
                    "config": {"workload": "chunked_ce fwd+grad", "rows": N, "hidden": H, "vocab": V,
                               "head": "int8 rows" if int8 else "bf16", "vocab_chunk": 32768, "token_chunk": tc},
                    "gpu_launches": launches,
                    "gemm_ms": round(gms, 3), "gemm_launches": gn,
                    "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": pk["bf16_tflops"],
                                 "unit": "TFLOP/s", "frac": round(tf / pk["bf16_tflops"], 3),
                                 "note": f"4 N V H flops (two GEMMs) over the whole step, {src} peak; GEMMs alone "
                                         f"{flops / (gms / 1e3) / 1e12:.0f} TFLOP/s"},
                    "cpu_baseline": cpu}
            print(json.dumps(line), flush=True)
        del head
        torch.cuda.empty_cache()


# ------------------------------------------------------------------------------------------ config 4 sweep
def run_sweep(args, local):
    """Config 4: the Qwen3.6 layer shape, forward only (no grad), all 256 experts frozen int4 group-64, at 1, 16, 128,
    1024 and 16384 tokens per call, routing uniform (router N(0, 0.02)) or Zipf s=1.2 (tau = 1). One JSON line per
    point with the achieved HBM bandwidth and tensor throughput over the algorithmic bytes and FLOPs of the call.
    Each call is a CUDA-graph replay timed alone between writes of a 256 MB buffer (L2 flushed)."""
    import smelb
    from smelb.synth import int4_bank_bytes_per_expert, qwen_layer
    dev = torch.device("cuda", local)
    H, E, K, I, S = 2048, 256, 8, 512, 512
    Ts = [1, 16, 128, 1024, 16384]
    pk, pk_kind = peaks()
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=dev)
    bank_b = int4_bank_bytes_per_expert(H, I)
    for routing in ("uniform", "zipf s=1.2"):
        L = qwen_layer(T=max(Ts), H=H, E=E, K=K, I=I, S=S, n_sel=0, with_lora=False, seed=4, device=dev,
                       uniform=routing == "uniform", zipf_s=1.2, tau=1.0)
        W, ex = L["W"], L["ex"]
        for T in Ts:
            x = L["x"][:T].contiguous()
            rec = {}
            with torch.no_grad():
                smelb.moe_forward(x, W, ex, K, None, stats=lambda p, v, i: rec.update(i=i))
            touched = int(torch.unique(rec["i"]).numel())
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side), torch.no_grad():
                for _ in range(3):
                    smelb.moe_forward(x, W, ex, K, None)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side), torch.no_grad():
                smelb.moe_forward(x, W, ex, K, None)
            torch.cuda.synchronize()
            ms = []
            for _ in range(max(args.steps, 5)):
                flush.fill_(1)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                ms.append(e0.elapsed_time(e1))
            t = statistics.median(ms) / 1e3
            nbytes = touched * bank_b + 3 * S * H * 2 + E * H * 2 + T * H * 2 * 2
            flops = T * (2 * K * 3 * H * I + 2 * 3 * H * S + 2 * H * E)
            gbs, tfl = nbytes / t / 1e9, flops / t / 1e12
            bound = "hbm" if nbytes / (pk["hbm_gbs"] * 1e9) > flops / (pk["bf16_tflops"] * 1e12) else "tensor"
            print(json.dumps({"sweep": "config 4 (forward only, all experts int4)", "tokens": T, "routing": routing,
                              "touched_experts": touched, "ms_per_call": round(t * 1e3, 4),
                              "tokens_per_s": round(T / t, 1), "algorithmic_bytes": nbytes, "hbm_gbs": round(gbs, 1),
                              "hbm_frac": round(gbs / pk["hbm_gbs"], 4), "tflops": round(tfl, 2),
                              "tc_frac": round(tfl / pk["bf16_tflops"], 4), "bound": bound,
                              "peaks": f"{pk_kind}: {pk['hbm_gbs']} GB/s, {pk['bf16_tflops']} TFLOP/s",
                              "timing": "median of graph replays, each after an L2 flush"}), flush=True)
            del g
            assert smelb.read_status() == 0


# ------------------------------------------------------------------------------------------ reference arm
def run_reference(args, world, rank):
    """The reference's CPU torch path (restated in oracle/cpu_step.py) on the host cores, same metric and config.
    The synthetic inputs come from the same seeded construction as our arm (smelb.synth.qwen_layer_tensors: torch
    operations only) with the bank quantized by the reference's algorithm (the oracle's quantizer, as torch
    operations); libsmelb is never loaded in this process. The timed steps run on the CPU alone."""
    if rank != 0:
        return None
    from oracle import cpu_step
    from smelb.synth import qwen_layer_tensors
    cfg = layer_config(args)
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    t = qwen_layer_tensors(T=cfg["T"], H=cfg["H"], E=cfg["E"], K=cfg["K"], I=cfg["I"], S=cfg["S"],
                           n_sel=cfg["n_sel"], r=cfg["r"], alpha=cfg["alpha"], seed=0, device=dev)
    torch.set_num_threads(os.cpu_count() or 1)
    tokens = min(cfg["T"], args.ref_tokens)
    p = cpu_step.prepare_tensors(t, dtype=torch.float32, tokens=tokens)
    meta = t["meta"]
    gy = torch.randn(p["x"].shape, generator=torch.Generator().manual_seed(9))
    del t
    if dev.type == "cuda":
        torch.cuda.empty_cache()
    times = []
    budget = args.ref_budget_s
    t_start = time.perf_counter()
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        cpu_step.step(p, gy)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
        if time.perf_counter() - t_start > budget and len(times) >= 1:
            break
    tot = sum(times)
    value = tokens * len(times) / tot
    res = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": len(times),
           "warmup": args.warmup, "ms_per_step": round(1e3 * tot / len(times), 2), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded)",
           "config": config_json(cfg, meta, world, args.parallel), "impl": "reference",
           "timing": "wall clock of the CPU steps (time.perf_counter)", "routing_share": round(meta.get("share", 0.0), 4),
           "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": torch.get_num_threads(),
                            "kind": "port", "cpu_model": cpu_model(),
                            "sample": f"{tokens} tokens per step, fp32 (the reference's faster CPU dtype), "
                                      f"{len(times)} timed steps"},
           "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=4092)
    ap.add_argument("--cpu-tokens", type=int, default=4092, help="tokens of the CPU-baseline sample")
    ap.add_argument("--ref-tokens", type=int, default=4092, help="tokens per reference-arm step")
    ap.add_argument("--ref-budget-s", type=float, default=150.0, help="stop the reference arm after this long")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="config 4 token-count sweep (one JSON line per point)")
    ap.add_argument("--stream", action="store_true",
                    help="layer-major forward over a stack of layers streamed from pinned host memory vs resident")
    ap.add_argument("--ce", action="store_true",
                    help="chunked cross-entropy over the Qwen3.6 LM head (one JSON line per head / chunking)")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 5],
                    help="2: the Qwen3.6 layer (default), 3: the Gemma 4 block, 5: the 24-layer layer-major block")
    ap.add_argument("--parallel", default="ep", choices=["dp", "ep"],
                    help="with N > 1: experts split over the GPUs (ep, the default) or data-parallel replicas (dp)")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    try:
        if args.sweep or args.stream or args.ce:
            if rank == 0:
                (run_sweep if args.sweep else run_stream if args.stream else run_ce)(args, local)
            res = None
        elif args.impl == "reference":
            res = run_reference(args, world, rank)
        elif args.config == 3:
            res = run_gemma(args, local) if rank == 0 else None
        elif args.config == 5:
            res = run_block(args, world, rank, local)
        else:
            res = run_ours(args, world, rank, local)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
