#!/usr/bin/env python3
"""Benchmark of the B200 GQA attention path (qx_b200 / libqxcuda).

Default workload (the metric's configuration): the Granite
24-layer attention-only decode stack, batch 1, fp32 KV, context 4096. The
cache holds 4032 synthetic rows; each step decodes one token through all 24
layers at positions 4032..4095 (RoPE, append, attention over 4033..4096
rows), cycling back to 4032 every 64 steps (cursor rollback, as the
reference's speculative rollback does), so every step reads ~400 MB of KV,
far more than the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config1|config0|config2|config3|config4|layer|commit|verify|sweep]

Prints one JSON line on rank 0 (`sweep`: one per context 512/2048/4096). N>1
runs under torchrun: one independent sequence (replica) per GPU, no
collective on the data path ("weak" scaling), device time max-reduced over
ranks. The config-1 line also carries `sharded`: config 4 (256 sequences)
sharded over the N ranks by LPT on KV bytes, with the one-GPU value of the
same run and the efficiency against N times it; at N>1 also `kv_split`:
config 3's single 32768-position context with its KV length split over the
ranks, the (m, l, O) partials crossing NVLink inside the decode grid, with
the one-GPU value of the same run. `--impl reference` times the CPU
restatement of qx's GQA path (oracle/, the reference being Rust and not
buildable here) with all host threads on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS = 24
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
# nominal B200 peaks, the denominators the north star quotes beside the measured ones
NOMINAL_HBM_GBS = 8000.0
NOMINAL_BF16_TFLOPS = 2250.0


def hbm_peak():
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(workload: str):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload)
    except Exception:
        return None


class ClockSampler:
    """Polls SM clock and throttle reasons through NVML while running."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle"}

    def __init__(self, device: int, period_s: float = 0.01):
        self.device, self.period = device, period_s
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            idx = self.device
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                idx = int(vis.split(",")[self.device])
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # no NVML: report nothing rather than guess
            self.error = str(e)
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def allreduce_max(value: float, world: int, device) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------------------------------
# config 1: Granite 24-layer stack, fp32 KV, batch 1
# ---------------------------------------------------------------------------------------
def granite_stack_bytes(attend: int, layers: int = LAYERS, s_kv: int = 4) -> int:
    """Algorithmic bytes of one decode step: per layer each cache row read
    once, the new row written once, q/k/v read and o written (f32):
    2*L*Hkv*d*s_kv + 4*d*(2*Hq + 2*Hkv)."""
    return layers * (2 * attend * 8 * 64 * s_kv + 4 * 64 * (2 * 16 + 2 * 8))


def run_config1(args, world, rank, local):
    import torch
    from qx_b200 import F32, MODEL_GRANITE, Context, KvArena
    from qx_b200 import _lib
    import ctypes as C

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = args.context
    cycle = 64
    P = L - cycle
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    arena = KvArena(ctx, MODEL_GRANITE, LAYERS, 1, L, F32, F32)
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580100 + rank)
    with torch.cuda.stream(stream):
        for l in range(LAYERS):
            arena.tensor(0, l, True)[:P].normal_(generator=g)
            arena.tensor(0, l, False)[:P].normal_(generator=g)
        q = torch.randn(cycle, LAYERS, 1024, device=dev, generator=g)
        k = torch.randn(cycle, LAYERS, 512, device=dev, generator=g)
        v = torch.randn(cycle, LAYERS, 512, device=dev, generator=g)
        out = torch.zeros(cycle, LAYERS, 1024, device=dev)
    stream.synchronize()
    arena.set_len(0, P)

    lib = ctx.lib
    flags = _lib.DECODE_NATIVE_EXP if args.native_exp else 0
    pos_arr = [(C.c_int32 * 1)(P + i) for i in range(cycle)]
    dargs = [_lib.DecodeArgs(0, LAYERS, 1, None, pos_arr[i], q[i].data_ptr(), k[i].data_ptr(), v[i].data_ptr(),
                             out[i].data_ptr(), None, None, None, F32, F32, F32, flags, args.split)
             for i in range(cycle)]
    dptrs = [C.byref(a) for a in dargs]

    def step(i):
        j = i % cycle
        if j == 0 and i > 0:
            arena.rollback(0, P)
        st = lib.qxc_decode(ctx.handle, arena.handle, dptrs[j])
        if st != 0:
            raise RuntimeError(lib.qxc_last_error(ctx.handle).decode())

    # warm-up (also brings the cursor to a known phase)
    arena.rollback(0, P)
    for i in range(args.warmup):
        step(i)
    ctx.sync()
    arena.rollback(0, P)
    barrier(world)

    K = args.steps
    # two events around the K steps and none between them (see timed_steps)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ctx.launch_count
    torch.cuda.synchronize(dev)
    barrier(world)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(K):
            step(i)
        end.record(stream)
        stream.synchronize()
    launches = ctx.launch_count - launches0
    split_used = ctx.last_split
    total_ms = start.elapsed_time(end)
    kernel_ms = [total_ms / K] * K  # one launch per step: its share of the timed region
    total_ms = allreduce_max(total_ms, world, dev)
    barrier(world)

    # algorithmic bytes per launch (one launch = one 24-layer step)
    attends = [P + (i % cycle) + 1 for i in range(K)]
    bytes_per_launch = [granite_stack_bytes(a) for a in attends]
    avg_bytes = float(np.mean(bytes_per_launch))
    avg_kernel_s = float(np.mean(kernel_ms)) / 1e3
    achieved_gbs = avg_bytes / avg_kernel_s / 1e9
    peak, peak_kind = hbm_peak()

    # e2e through the public host-buffer API (qxc_decode_host)
    e2e = None
    if not args.no_e2e:
        # the step's inputs and output live in pinned host memory
        hq = q.cpu().pin_memory().numpy()
        hk = k.cpu().pin_memory().numpy()
        hv = v.cpu().pin_memory().numpy()
        hout = torch.zeros(LAYERS, 1024).pin_memory().numpy()
        hpos = [(C.c_int32 * 1)(P + i) for i in range(cycle)]
        hargs = [_lib.DecodeArgs(0, LAYERS, 1, None, hpos[i], hq[i].ctypes.data, hk[i].ctypes.data,
                                 hv[i].ctypes.data, hout.ctypes.data, None, None, None, F32, F32, F32, flags, args.split)
                 for i in range(cycle)]
        hptr = [C.byref(a) for a in hargs]
        E = min(K, args.e2e_steps)

        def hstep(i):
            j = i % cycle
            if j == 0 and i > 0:
                arena.rollback(0, P)
            st = lib.qxc_decode_host(ctx.handle, arena.handle, hptr[j])
            if st != 0:
                raise RuntimeError(lib.qxc_last_error(ctx.handle).decode())

        arena.rollback(0, P)
        for i in range(min(args.warmup, cycle)):
            hstep(i)
        arena.rollback(0, P)
        barrier(world)
        t0 = time.perf_counter()
        for i in range(E):
            hstep(i)
        e2e_s = allreduce_max(time.perf_counter() - t0, world, dev)
        e2e = {"value": world * E / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": LAYERS * (1024 + 512 + 512) * 4,
               "d2h_bytes_per_step": LAYERS * 1024 * 4, "steps": E,
               "api": "qxc_decode_host (pinned host q/k/v in, pinned host out, synchronous)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_config1(L, threads=1, steps=args.cpu_steps)

    traffic = profile_traffic("config1")
    line = {
        "metric": "attention-stack decode tok/s (Granite 24-layer GQA stack, batch 1 per GPU)",
        "value": world * K / (total_ms / 1e3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": total_ms / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded N(0,1) q/k/v and KV cache (torch.Generator on device)",
        "config": {"workload": f"config1: Granite-3.0-1B-A400M attention stack, 24 layers, fp32 KV, context {L}, "
                               f"positions {P}..{L - 1} cycled, batch 1",
                   "context": L, "layers": LAYERS, "kv_dtype": "f32", "batch_per_gpu": 1,
                   "l2": "inputs larger than L2: each step reads ~%.0f MB of KV" % (avg_bytes / 1e6),
                   "parallelism": f"replicas x{world} (independent sequences, no collective)",
                   "softmax_exp": "native exp2" if args.native_exp else "qx pinned exp_f32",
                   "split": split_used},
        "hbm_gbs": achieved_gbs,
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                     "frac": achieved_gbs / peak, "peak_kind": peak_kind,
                     "frac_of_nominal": achieved_gbs / NOMINAL_HBM_GBS,
                     "traffic": traffic["bytes_per_launch"] if traffic else None,
                     "kernel": "qx_decode_kernel<Granite,float,float>",
                     "algorithmic_bytes_per_launch": avg_bytes, "avg_launch_us": avg_kernel_s * 1e6},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if e2e:
        line["e2e"] = e2e
    if cpu:
        line["cpu_baseline"] = cpu
    arena.close()
    ctx.close()
    return line


def cpu_baseline_config1(L, threads, steps):
    """The oracle (C restatement of qx-runtime's granite_attention_decode)
    timed on this host: `steps` full 24-layer steps at attended length ~L."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle as o
    from qx_b200 import synthetic as syn
    o.build()
    P = L - 1
    kc = syn.normal(11, (P, 8, 64))
    vc = syn.normal(12, (P, 8, 64))
    caches = []
    for _ in range(LAYERS):
        c = o.KvCache(L)
        c.keys[:P], c.values[:P] = kc, vc
        caches.append(c)
    qs = [syn.normal(13 + l, (1024,)) for l in range(LAYERS)]
    ks = [syn.normal(113 + l, (512,)) for l in range(LAYERS)]
    vs = [syn.normal(213 + l, (512,)) for l in range(LAYERS)]
    t0 = time.perf_counter()
    for _ in range(steps):
        for c in caches:
            c.length.value = P
        worst, _ = o.granite_decode_many(qs, ks, vs, [P] * LAYERS, caches, threads=threads)
        assert worst == 0
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{steps} full 24-layer decode steps at context {L}, {threads} thread(s), "
                      "oracle/qx_oracle.c (restatement of qx-runtime granite_attention_decode)",
            "seconds": dt}


# ---------------------------------------------------------------------------------------
# shared timing harness for the other workloads
# ---------------------------------------------------------------------------------------
def tensor_peak():
    try:
        with open(PEAKS_PATH) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def timed_steps(step, K, W, stream, world, dev, local, ctx):
    """W warm-up then K timed steps between two CUDA events on `stream`;
    returns (max-over-ranks total ms, per-step ms list, clocks, launches).
    No event sits between the steps: consecutive launches overlap their
    set-up with the previous grid's tail (programmatic dependent launch),
    which an event recorded between them would prevent. A step's time is
    its share of the timed region, total / K."""
    import torch
    for i in range(W):
        step(i)
    stream.synchronize()
    ctx.sync()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ctx.launch_count
    torch.cuda.synchronize(dev)
    barrier(world)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(K):
            step(W + i)
        end.record(stream)
        stream.synchronize()
    ctx.sync()
    local_ms = start.elapsed_time(end)
    total = allreduce_max(local_ms, world, dev)
    return total, [local_ms / K] * K, clk.summary(), ctx.launch_count - launches0


def base_line(metric, value, unit, world, K, W, total_ms, higher, scaling, dtype, config, clocks, launches):
    return {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": total_ms / K, "higher_is_better": higher, "scaling": scaling, "vs_baseline": None,
            "dtype": dtype, "data": "synthetic: seeded N(0,1)", "config": config, "clocks": clocks,
            "gpu_launches": int(launches)}


def hbm_roofline(bytes_per_launch, per_ms, kernel, workload=None):
    """`traffic` is the ncu DRAM read+write of one launch of the same
    workload (profiles/traffic.json), when one was captured."""
    peak, kind = hbm_peak()
    ach = bytes_per_launch / (float(np.mean(per_ms)) / 1e3) / 1e9
    tr = profile_traffic(workload) if workload else None
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "peak_kind": kind,
            "frac_of_nominal": ach / NOMINAL_HBM_GBS, "traffic": (tr["dram_read"] + tr["dram_write"]) if tr else None, "kernel": kernel,
            "algorithmic_bytes_per_launch": bytes_per_launch, "avg_launch_us": float(np.mean(per_ms)) * 1e3}


def run_config0(args, world, rank, local):
    """Config 0: one Granite layer, fp32, 511 cached rows + the new token at 511."""
    import torch
    from qx_b200 import F32, MODEL_GRANITE, Context, KvArena
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    # the calls rotate over NSET copies of the config (2.1 MB each, 168 MB in
    # all, beyond the 126 MB L2), so no call finds its cache in L2
    NSET = 80
    arena = KvArena(ctx, MODEL_GRANITE, 1, NSET, 512, F32, F32)
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580000)
    with torch.cuda.stream(stream):
        for s in range(NSET):
            arena.tensor(s, 0, True)[:511].normal_(generator=g)
            arena.tensor(s, 0, False)[:511].normal_(generator=g)
        q = torch.randn(1, 1024, device=dev, generator=g)
        k = torch.randn(1, 512, device=dev, generator=g)
        v = torch.randn(1, 512, device=dev, generator=g)
        out = torch.zeros(1, 1024, device=dev)
    stream.synchronize()

    def one(i):
        arena.set_len(i % NSET, 511)
        arena.decode(q, k, v, out, [511], seq_ids=[i % NSET], split=args.split)

    # A single call is a few microseconds of GPU work, less than the host's
    # launch path, so the calls are captured in a CUDA graph (R per replay)
    # and the graph is replayed: the timing is then the device's own.
    R = 100
    for i in range(3):
        one(i)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(R):
            one(i)

    def step(i):
        graph.replay()

    K, W = max(1, args.steps // R), max(3, args.warmup // R)
    with torch.cuda.stream(stream):  # graph.replay() launches on the current stream
        total, per, clk, launches = timed_steps(step, K, W, stream, world, dev, local, ctx)
    launches = K * R
    per = [x / R for x in per]  # per call
    K = K * R                   # total covers all K * R calls
    B = 2 * 512 * 8 * 64 * 4 + 4 * 64 * (2 * 16 + 2 * 8)
    us = float(np.mean(per)) * 1e3
    line = base_line("single-layer Granite GQA decode latency (us per call)", us, "us", world, K, W, total, False,
                     "weak", "f32", {"workload": "config0: Granite 1 layer, fp32 KV, 511 cached + new token at 511",
                                     "l2": "calls rotate over 80 cache copies (168 MB > 126 MB L2)",
                                     "timing": "100 calls per CUDA graph replay; per-call device time"}, clk, launches)
    line["roofline"] = hbm_roofline(B, per, "qx_decode_kernel<Granite,float,float>")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import py_oracle as o
        from qx_b200 import synthetic as syn
        o.build()
        c = o.KvCache(512)
        c.keys[:511] = syn.normal(1, (511, 8, 64))
        c.values[:511] = syn.normal(2, (511, 8, 64))
        qq, kk, vv = syn.normal(3, (1024,)), syn.normal(4, (512,)), syn.normal(5, (512,))
        n = 200
        t0 = time.perf_counter()
        for _ in range(n):
            c.length.value = 511
            o.granite_attention_decode(qq, kk, vv, 511, c)
        dt = (time.perf_counter() - t0) / n
        line["cpu_baseline"] = {"value": dt * 1e6, "unit": "us", "cores": 1, "kind": "port",
                                "sample": f"{n} calls of the oracle granite_attention_decode at context 512"}
    arena.close()
    ctx.close()
    return line


def run_config2(args, world, rank, local):
    """Config 2: Granite causal prefill, bf16 in, f32 accumulate, L = --context (512 or 2048)."""
    import torch
    from qx_b200 import BF16, MODEL_GRANITE, Context, KvArena
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = args.prefill_len
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    # the calls rotate over NSET independent prompts (q/k/v in, cache and f32
    # output out: 12 KB per position), together beyond the 126 MB L2
    NSET = max(2, -(-160 * 2**20 // (12288 * L)))
    arena = KvArena(ctx, MODEL_GRANITE, 1, NSET, L, BF16, BF16)
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580200)
    with torch.cuda.stream(stream):
        q = (torch.randn(NSET, L, 16, 64, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        k = (torch.randn(NSET, L, 8, 64, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        v = (torch.randn(NSET, L, 8, 64, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        out = torch.zeros(NSET, L, 16, 64, device=dev)
    stream.synchronize()

    def one(i):
        s = i % NSET
        arena.reset(s)
        arena.prefill(q[s], k[s], v[s], out[s], L, seq=s)

    # the host path of one call (three tensor-map encodes, argument checks)
    # takes longer than the GPU work at these lengths: capture R calls in a
    # CUDA graph and time its replays, so the numbers are device time
    R = 20
    for i in range(3):
        one(i)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(R):
            one(i)

    def step(i):
        graph.replay()

    K, W = max(1, args.steps // R), max(3, args.warmup // R)
    with torch.cuda.stream(stream):
        total, per, clk, launches = timed_steps(step, K, W, stream, world, dev, local, ctx)
    per = [x / R for x in per]  # per call
    launches = K * R * 2
    K *= R
    flops = 2 * 16 * 64 * L * (L + 1)
    peak, kind = tensor_peak()
    ach = flops / (float(np.mean(per)) / 1e3) / 1e12
    line = base_line("Granite causal GQA prefill TFLOP/s", world * flops * K / (total / 1e3) / 1e12, "TFLOP/s",
                     world, K, W, total, True, "weak", "bf16",
                     {"workload": f"config2: Granite causal prefill, L={L}, 16/8 heads, d=64, bf16 in, f32 acc",
                      "l2": f"calls rotate over {NSET} prompts ({NSET * 12288 * L / 2**20:.0f} MB > 126 MB L2)",
                      "timing": "20 calls per CUDA graph replay",
                      "flops_per_step": flops}, clk, launches)
    line["roofline"] = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                        "peak_kind": kind, "frac_of_nominal": ach / NOMINAL_BF16_TFLOPS,
                        "traffic": (lambda t: t["dram_read"] + t["dram_write"] if t else None)(
                            profile_traffic(f"config2_l{L}")),
                        "kernel": "qx_prefill_rope_kernel + qx_prefill_attn_tc_kernel (timed together)",
                        "algorithmic_flops_per_launch": flops, "avg_launch_us": float(np.mean(per)) * 1e3}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import py_oracle as o
        from qx_b200 import synthetic as syn
        o.build()
        Ls = 512
        qs = syn.to_bf16_bits(syn.normal(1, (Ls, 16, 64), 0.5))
        ks = syn.to_bf16_bits(syn.normal(2, (Ls, 8, 64), 0.5))
        vs = syn.to_bf16_bits(syn.normal(3, (Ls, 8, 64), 0.5))
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        o.granite_prefill(qs, ks, vs, o.BF16, o.BF16, threads=threads)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": 2 * 16 * 64 * Ls * (Ls + 1) / dt / 1e12, "unit": "TFLOP/s",
                                "cores": threads, "kind": "port",
                                "sample": f"oracle prefill (iterated decode) at L={Ls} on {threads} threads"}
    arena.close()
    ctx.close()
    return line


def run_config3(args, world, rank, local):
    """Config 3: Qwen3 attention decode, bf16 KV, KV length 32768; N>1 splits the KV length."""
    import torch
    from qx_b200 import BF16, MODEL_QWEN3, Context, KvArena
    from qx_b200.distributed import all_gather_partials, kv_ranges, open_peer_group
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = args.qwen_context
    P = L - 1
    b, e = kv_ranges(L, world)[rank]
    owner = rank == world - 1
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    # the calls rotate over NSET copies of this rank's cache, together beyond
    # the 126 MB L2, so no call finds its cache in L2
    NSET = max(2, -(-192 * 2**20 // (2 * (e - b) * 4 * 128 * 2)))
    arena = KvArena(ctx, MODEL_QWEN3, 1, NSET, e - b, BF16, BF16, first_position=b)
    cached = min(e, P) - b
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580300 + rank)
    with torch.cuda.stream(stream):
        for s in range(NSET):
            arena.tensor(s, 0, True)[:cached].view(torch.bfloat16).normal_(generator=g)
            arena.tensor(s, 0, False)[:cached].view(torch.bfloat16).normal_(generator=g)
        gq = torch.Generator(device=dev)
        gq.manual_seed(0x51580301)  # q/k/v identical on every rank
        q = torch.randn(1, 4096, device=dev, generator=gq).to(torch.bfloat16)
        k = torch.randn(1, 512, device=dev, generator=gq).to(torch.bfloat16)
        v = torch.randn(1, 512, device=dev, generator=gq).to(torch.bfloat16)
        out = torch.zeros(1, 4096, device=dev)
        parts = torch.zeros(32, 130, device=dev)
        merged = torch.zeros(4096, device=dev)
    stream.synchronize()
    for s in range(NSET):
        arena.set_len(s, cached)
    # N>1: the partials cross NVLink through qxc_exchange_merge (peer stores
    # into every rank's area + merge, one kernel), or with --exchange nccl
    # through an NCCL all-gather and qxc_lse_merge
    peers = open_peer_group(ctx) if world > 1 and args.exchange in ("peer", "kernel") else None

    def step(i):
        s = i % NSET
        if world == 1:
            arena.set_len(s, P)
            arena.decode(q, k, v, out, [P], seq_ids=[s], split=args.split)
            return
        arena.set_len(s, cached)
        if args.exchange == "peer":  # the exchange inside the split merge kernel
            arena.decode_exchange(q, k, v, merged, P, append=owner, group=peers, seq=s, split=args.split)
            return
        arena.decode_partials(q, k, v, parts, P, append=owner, seq=s, split=args.split)
        if peers is not None:
            peers.exchange_merge(MODEL_QWEN3, parts, merged)
        else:
            allp = all_gather_partials(parts)
            ctx.lse_merge(MODEL_QWEN3, world, allp, merged)

    K, W = args.steps, args.warmup
    # one step is tens of microseconds of GPU work, comparable to the host's
    # per-call path: capture R steps in a CUDA graph (the NCCL all-gather of
    # the N>1 path included) and replay it
    R = 50 if world == 1 else 20
    with torch.cuda.stream(stream):
        for i in range(3):
            step(i)
    stream.synchronize()
    barrier(world)
    graph = torch.cuda.CUDAGraph()
    n0 = ctx.launch_count
    with torch.cuda.graph(graph, stream=stream):
        for i in range(R):
            step(i)
    per_replay = ctx.launch_count - n0  # our kernels in one replay
    replay = lambda i: graph.replay()  # noqa: E731
    K, W = max(1, K // R), max(3, W // R)
    with torch.cuda.stream(stream):
        total, per, clk, launches = timed_steps(replay, K, W, stream, world, dev, local, ctx)
    stream.synchronize()
    del graph  # a graph holding NCCL work must go before the process group
    if peers is not None:
        barrier(world)  # no rank closes its area while a peer may still store into it
        peers.close()
    per = [x / R for x in per]  # per call
    launches = K * per_replay
    K *= R                          # total covers all K * R calls
    B = 2 * L * 4 * 128 * 2 + 4 * 128 * (2 * 32 + 2 * 4)
    per_rank_bytes = 2 * (e - b) * 4 * 128 * 2
    line = base_line("Qwen3-30B-A3B attention decode tok/s (KV 32768, bf16)", K / (total / 1e3), "tok/s", world, K,
                     W, total, True, "strong", "bf16",
                     {"workload": "config3: Qwen3 layer decode, 32 q / 4 kv heads, d=128, bf16 KV, length 32768",
                      "l2": f"calls rotate over {NSET} cache copies ({NSET * per_rank_bytes / 2**20:.0f} MB > 126 MB L2)",
                      "parallelism": "single GPU" if world == 1 else
                      {"peer": f"KV length split x{world}; the decode grid merges its splits and pushes each "
                               "rank's (m,l,O) slices to every rank with tagged NVLink peer stores, then merges "
                               "the ranks' slices (qxc_decode_exchange)",
                       "kernel": f"KV length split x{world}; (m,l,O) partials exchanged with NVLink peer stores "
                                 "and merged by a separate kernel (qxc_exchange_merge)",
                       "nccl": f"KV length split x{world}, NCCL all-gather of (m,l,O) partials + LSE merge"}
                      [args.exchange],
                      "timing": f"{R} steps per CUDA graph replay"},
                     clk, launches)
    line["config"]["split"] = ctx.last_split
    kernel = ("qx_decode_tc_kernel<bf16,TcQwen> (splits merged inside the grid)" if world == 1 else
              {"peer": "qx_decode_tc_kernel<bf16,TcQwen> (splits merged and exchanged over NVLink inside the grid)",
               "kernel": "qx_decode_tc_kernel<bf16,TcQwen> + qx_exchange_merge_kernel (timed together)",
               "nccl": "qx_decode_tc_kernel<bf16,TcQwen> + NCCL all-gather + qx_lse_merge_kernel (timed together)"}
              [args.exchange])
    line["roofline"] = hbm_roofline(B if world == 1 else per_rank_bytes, per, kernel,
                                    "config3" if world == 1 else None)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import py_oracle as o
        from qx_b200 import synthetic as syn
        o.build()
        conv = syn.to_bf16_bits
        qb_, kb_, vb_ = conv(syn.normal(1, (32, 128))), conv(syn.normal(2, (4, 128))), conv(syn.normal(3, (4, 128)))
        kc = conv(syn.normal(4, (L, 4, 128)))  # same length as the GPU run
        vc = conv(syn.normal(5, (L, 4, 128)))
        ones = np.ones(128, np.float32)
        t0 = time.perf_counter()
        o.qwen_decode(qb_, kb_, vb_, ones, ones, kc, vc, P, o.BF16, threads=1)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": 1.0 / dt, "unit": "tok/s", "cores": 1, "kind": "port",
                                "sample": "one oracle Qwen decode step (qk-norm RoPE, store, GQA over 32768)"}
    arena.close()
    ctx.close()
    return line


def run_layer(args, world, rank, local):
    """The attention sub-layers of the Granite stack with Q4 weights (the
    reference's --v2-attention-stack: PreparedAttentionStack::encode runs
    encode_attention_layer for each of the 24 layers, the hidden state
    chained from layer to layer: RMSNorm, Q4 q/k/v, RoPE + append +
    attention, Q4 o-projection, residual), fp32 KV at context --context,
    positions cycled over the last 64 like config 1. One qxc_attention_stack
    call per token (one persistent launch for all 24 layers); with
    --layer-chain, qxc_attention_layer per layer instead (four launches per
    layer, captured in a CUDA graph). Random Q4 codes and FP16 scales stand
    in for the .qx weights."""
    import torch
    from qx_b200 import F32, MODEL_GRANITE, Context, KvArena, Q4Weights
    from qx_b200 import _lib
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = args.context
    cycle = 64
    P = L - cycle
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    arena = KvArena(ctx, MODEL_GRANITE, LAYERS, 1, L, F32, F32)
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580500 + rank)

    def q4w(rows, cols):
        codes = torch.randint(0, 255, (rows, cols // 32, 16), dtype=torch.uint8, device=dev, generator=g)
        scales = (torch.rand(rows, cols // 32, device=dev, generator=g) * 0.004 + 0.001).to(torch.float16)
        return Q4Weights(codes, scales.view(torch.int16), rows, cols)

    with torch.cuda.stream(stream):
        for l in range(LAYERS):
            arena.tensor(0, l, True)[:P].normal_(generator=g)
            arena.tensor(0, l, False)[:P].normal_(generator=g)
        weights = [dict(norm=1.0 + 0.1 * torch.randn(1024, device=dev, generator=g), q=q4w(1024, 1024),
                        k=q4w(512, 1024), v=q4w(512, 1024), o=q4w(1024, 1024)) for _ in range(LAYERS)]
        hidden = [torch.randn(1024, device=dev, generator=g) for _ in range(2)]
    stream.synchronize()
    arena.set_len(0, P)

    if args.layer_chain:
        def one(i):
            pos = P + i % cycle
            for l in range(LAYERS):
                w = weights[l]
                arena.attention_layer(hidden[l % 2], hidden[(l + 1) % 2], w["norm"], w["q"], w["k"], w["v"],
                                      w["o"], pos, layer=l, flags=_lib.DECODE_NO_ADVANCE if l + 1 < LAYERS else 0,
                                      split=args.split)

        # one step is 72 launches of a few microseconds each: capture a whole
        # cycle of 64 tokens in a CUDA graph and replay it (the host cursor is
        # rewound before each replay; the graph's kernels carry their positions)
        with torch.cuda.stream(stream):
            for i in range(3):
                one(i)
        stream.synchronize()
        arena.rollback(0, P)
        graph = torch.cuda.CUDAGraph()
        n0 = ctx.launch_count
        with torch.cuda.graph(graph, stream=stream):
            for i in range(cycle):
                one(i)
        per_replay = ctx.launch_count - n0

        def replay(i):
            arena.rollback(0, P)
            graph.replay()

        K, W = max(1, args.steps // cycle), max(3, args.warmup // cycle)
        with torch.cuda.stream(stream):
            total, per, clk, _ = timed_steps(replay, K, W, stream, world, dev, local, ctx)
        stream.synchronize()
        per = [x / cycle for x in per]  # per token
        steps = K * cycle
        launches = K * per_replay
        kernel = "qx_q4_matvec_kernel + qx_decode_kernel<Granite,float,float> + qx_split_merge_kernel"
        timing = "64 tokens per CUDA graph replay"
    else:
        import ctypes as C
        # the call's arguments, built once per position (the host cost per
        # token is then one ctypes call)
        ws = (_lib.LayerWeights * LAYERS)()
        for l, w in enumerate(weights):
            ws[l] = _lib.LayerWeights(w["norm"].data_ptr(), w["q"].ref(), w["k"].ref(), w["v"].ref(), w["o"].ref())
        sargs = [_lib.StackArgs(0, 0, LAYERS, P + j, hidden[0].data_ptr(), hidden[1].data_ptr(), ws, 0, args.split)
                 for j in range(cycle)]
        sptr = [C.byref(a) for a in sargs]
        lib = ctx.lib

        def one(i):
            j = i % cycle
            if j == 0 and i > 0:
                arena.rollback(0, P)
            st = lib.qxc_attention_stack(ctx.handle, arena.handle, sptr[j])
            if st != 0:
                raise RuntimeError(lib.qxc_last_error(ctx.handle).decode())

        arena.rollback(0, P)
        K, W = args.steps, args.warmup
        total, per, clk, launches = timed_steps(one, K, W, stream, world, dev, local, ctx)
        steps = K
        kernel = "qx_attention_stack_kernel"
        timing = "one qxc_attention_stack call (one launch) per token"
    kv = sum(granite_stack_bytes(P + j + 1) for j in range(cycle)) / cycle
    wbytes = LAYERS * (1024 + 512 + 512 + 1024) * (1024 // 2 + 1024 // 32 * 2)
    B = kv + wbytes + LAYERS * 2 * 1024 * 4 * 2
    line = base_line("attention sub-layer stack tok/s (Granite 24 layers, Q4 projections, fp32 KV)",
                     world * steps / (total / 1e3), "tok/s", world, steps, W, total, True, "weak", "f32",
                     {"workload": f"Granite 24-layer attention sub-layers with Q4 q/k/v/o (random codes), fp32 KV, "
                                  f"context {L}, positions {P}..{L - 1} cycled, batch 1",
                      "l2": "inputs larger than L2: ~400 MB of KV and 42 MB of Q4 weights per token",
                      "timing": timing, "bytes_per_token": int(B), "split": ctx.last_split},
                     clk, launches)
    line["roofline"] = hbm_roofline(B, per, kernel, None if args.layer_chain or L != 4096 else "layer")
    arena.close()
    ctx.close()
    return line


def run_commit(args, world, rank, local):
    """KV-slot commitments (the reference's verification-hash stage): every
    step hashes all 24 x 4096 slots of an fp32 Granite cache (402 MB, more
    than the 126 MB L2) into 98,304 kv_leaf_hash_v1 digests with one
    qxc_kv_slot_hashes launch; the per-token call of the reference
    (qxc_verification_hashes: 25 positions, state roots + slot leaves) is
    timed beside it. BLAKE3 is integer-ALU work: the roofline is the
    measured compress-only rate of the same compression function."""
    import torch
    from qx_b200 import F32, MODEL_GRANITE, Context, KvArena
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L = args.context
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    arena = KvArena(ctx, MODEL_GRANITE, LAYERS, 1, L, F32, F32)
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580600 + rank)
    slots = LAYERS * L
    with torch.cuda.stream(stream):
        for l in range(LAYERS):
            arena.tensor(0, l, True).normal_(generator=g)
            arena.tensor(0, l, False).normal_(generator=g)
        digests = torch.zeros(LAYERS, L, 32, dtype=torch.uint8, device=dev)
        residuals = torch.randn(LAYERS + 1, 1024, device=dev, generator=g)
        vdig = torch.zeros(LAYERS + 1, 64, dtype=torch.uint8, device=dev)
    stream.synchronize()
    arena.set_len(0, L)

    def step(i):
        arena.slot_hashes(digests, 0, LAYERS, 0, L)

    with torch.cuda.stream(stream):
        total, per, clk, launches = timed_steps(step, args.steps, args.warmup, stream, world, dev, local, ctx)
    stream.synchronize()
    K = args.steps
    rate = ctx.blake3_compress_rate()
    per_slot = 5 * 16 + 7 + 7 + 2  # leaves of 8 key + 8 value chunks, two 8-leaf trees, the 2-block slot leaf
    avg_s = float(np.mean(per)) / 1e3
    ach = slots * per_slot / avg_s
    line = base_line("KV slot commitments/s (BLAKE3 kv_leaf_hash_v1, Granite 24 layers x 4096 tokens, fp32 KV)",
                     world * K * slots / (total / 1e3), "slots/s", world, K, args.warmup, total, True, "weak", "u32",
                     {"workload": f"all {LAYERS} x {L} (layer, token) slots of one fp32 Granite KV cache per step "
                                  "(2 KB key + 2 KB value rows), one launch",
                      "l2": f"inputs larger than L2: {slots * 4096 / 1e6:.0f} MB of KV hashed per step",
                      "bytes_per_slot": 4096, "compressions_per_slot": per_slot},
                     clk, launches)
    # ncu DRAM bytes of a 24 x 2048-slot launch, scaled by the slots hashed
    tr = profile_traffic("commit_ctx2048")
    traffic = (tr["dram_read"] + tr["dram_write"]) * slots / tr["slots_per_launch"] if tr else None
    line["roofline"] = {"bound": "alu", "achieved": ach / 1e9, "peak": rate / 1e9, "unit": "Gcompress/s",
                        "frac": ach / rate, "peak_kind": "measured (qxc_blake3_compress_rate: the same BLAKE3 "
                                                         "compression, registers only, every SM)",
                        "traffic": traffic, "kernel": "qx_kv_hash_serial_kernel",
                        "hbm_GBps": slots * 4096 / avg_s / 1e9, "avg_launch_us": avg_s * 1e6}
    # the reference's per-token call: 25 positions (genesis + 24 layers),
    # 4 KB residual snapshots, checkpoint interval 1 (its default)
    with torch.cuda.stream(stream):
        for _ in range(5):
            arena.verification_hashes(L - 1, residuals, 4096, 1, vdig)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(200):
            arena.verification_hashes(L - 1, residuals, 4096, 1, vdig)
        e1.record(stream)
    stream.synchronize()
    line["per_token_call_us"] = e0.elapsed_time(e1) / 200 * 1e3
    # the lane-per-chunk layout on the same range (the small-range default)
    from qx_b200 import HASH_PER_CHUNK
    with torch.cuda.stream(stream):
        for _ in range(3):
            arena.slot_hashes(digests, 0, LAYERS, 0, L, layout=HASH_PER_CHUNK)
        e0.record(stream)
        for _ in range(10):
            arena.slot_hashes(digests, 0, LAYERS, 0, L, layout=HASH_PER_CHUNK)
        e1.record(stream)
    stream.synchronize()
    line["per_chunk_layout_slots_per_s"] = slots * 10 / (e0.elapsed_time(e1) / 1e3)
    # e2e: the public call plus the digests read back to pinned host memory
    # (the hashed rows are the resident cache itself, nothing is uploaded)
    if not args.no_e2e:
        host = torch.empty(digests.shape, dtype=torch.uint8).pin_memory()
        E = max(3, K // 4)

        def estep(i):
            arena.slot_hashes(digests, 0, LAYERS, 0, L)
            host.copy_(digests, non_blocking=True)

        with torch.cuda.stream(stream):
            et, _, _, _ = timed_steps(estep, E, args.warmup, stream, world, dev, local, ctx)
        line["e2e"] = {"value": world * E * slots / (et / 1e3), "unit": "slots/s", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": int(digests.numel())}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import py_oracle as o
        o.build()
        rows = [(arena.read(0, l, t, 1)) for l, t in ((l, t) for l in range(2) for t in range(64))]
        kb = [k.tobytes() for k, _ in rows]
        vb = [v.tobytes() for _, v in rows]
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0:
            for j in range(len(kb)):
                o.kv_leaf_hash(j // 64, j % 64, kb[j], vb[j])
            n += len(kb)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": n / dt, "unit": "slots/s", "cores": 1, "kind": "port",
                                "sample": f"{n} kv_leaf_hash_v1 slots of the same cache (fp32 rows), one thread, "
                                          "oracle/qx_oracle.c (restatement of qx-commit state.rs with the "
                                          "published BLAKE3)", "seconds": dt}
    arena.close()
    ctx.close()
    return line


def run_verify(args, world, rank, local):
    """Speculative verify (the reference's batched verifier stage): each step
    checks K = 4 candidate tokens of one sequence through the Granite
    24-layer stack, fp32 KV, context 4096, in one qxc_decode_verify call
    (the candidates' rows appended, token t attending [0, start + t]); the
    cursor then rolls back to the checkpoint, as after a rejected draft."""
    import torch
    from qx_b200 import F32, MODEL_GRANITE, Context, KvArena
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    L, Kc = args.context, 4
    P = L - Kc
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    arena = KvArena(ctx, MODEL_GRANITE, LAYERS, 1, L, F32, F32)
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580700 + rank)
    NSET = 16  # candidate sets, cycled
    with torch.cuda.stream(stream):
        for l in range(LAYERS):
            arena.tensor(0, l, True)[:P].normal_(generator=g)
            arena.tensor(0, l, False)[:P].normal_(generator=g)
        q = torch.randn(NSET, Kc, LAYERS, 1024, device=dev, generator=g)
        k = torch.randn(NSET, Kc, LAYERS, 512, device=dev, generator=g)
        v = torch.randn(NSET, Kc, LAYERS, 512, device=dev, generator=g)
        out = torch.zeros(Kc, LAYERS, 1024, device=dev)
    stream.synchronize()
    arena.set_len(0, P)

    def step(i):
        arena.rollback(0, P)
        j = i % NSET
        arena.decode_verify(q[j], k[j], v[j], out, P, Kc, split=args.split)

    with torch.cuda.stream(stream):
        total, per, clk, launches = timed_steps(step, args.steps, args.warmup, stream, world, dev, local, ctx)
    stream.synchronize()
    K = args.steps
    # algorithmic bytes: the cache read once (P + K rows per layer) and the
    # candidates' q/k/v/out; the K tokens share every row
    row = 8 * 64 * 4
    B = LAYERS * (2 * (P + Kc) * row + Kc * (1024 + 512 + 512 + 1024) * 4)
    line = base_line("speculative verify tok/s (Granite 24-layer stack, 4 candidates per step, fp32 KV)",
                     world * K * Kc / (total / 1e3), "tok/s", world, K, args.warmup, total, True, "weak", "f32",
                     {"workload": f"qxc_decode_verify of {Kc} candidate tokens at positions {P}..{L - 1} through "
                                  f"24 Granite layers, fp32 KV, context {L}, cursor rolled back after each step",
                      "l2": "inputs larger than L2: ~%.0f MB of KV per step" % (LAYERS * 2 * P * row / 1e6),
                      "candidates": Kc},
                     clk, launches)
    line["verify_steps_per_s"] = world * K / (total / 1e3)
    line["config"]["split"] = ctx.last_split
    line["roofline"] = hbm_roofline(B, per, "qx_append_rows_kernel + qx_verify_kernel<float,float> (timed together)",
                                    "verify" if L == 4096 else None)
    arena.close()
    ctx.close()
    return line


def config4_measure(args, local, lengths, mine, K, W, timing_world):
    """Decode one step of sequences `mine` (indices into `lengths`) through
    24 layers per timed step, bf16 KV; returns a dict of the measurement.
    `timing_world` ranks take part in the barriers and the max-reduce of the
    time (1: this rank alone)."""
    import ctypes as C
    import torch
    from qx_b200 import BF16, F32, MODEL_GRANITE, Context, KvArena
    from qx_b200 import _lib
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n = len(mine)
    ctx = Context(local)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream)
    page = args.paged
    g = torch.Generator(device=dev)
    g.manual_seed(0x51580401 + mine[0])
    if page:
        # a paged arena sized to the batch: each sequence maps ceil(L / page)
        # pages of the shared pool instead of a 4096-row cache per layer
        pool = sum((lengths[i] + page - 1) // page for i in mine)
        arena = KvArena(ctx, MODEL_GRANITE, LAYERS, n, 4096, BF16, BF16, page_size=page, pool_pages=pool)
        with torch.cuda.stream(stream):
            arena.pool_tensor(True).view(torch.bfloat16).normal_(generator=g)
            arena.pool_tensor(False).view(torch.bfloat16).normal_(generator=g)
        for s, i in enumerate(mine):
            arena.set_len(s, lengths[i])  # maps the pages
        kv_bytes = 2 * LAYERS * pool * page * 8 * 64 * 2
    else:
        arena = KvArena(ctx, MODEL_GRANITE, LAYERS, n, 4096, BF16, BF16)
        with torch.cuda.stream(stream):
            for s, i in enumerate(mine):
                for l in range(LAYERS):
                    arena.tensor(s, l, True)[:lengths[i] - 1].view(torch.bfloat16).normal_(generator=g)
                    arena.tensor(s, l, False)[:lengths[i] - 1].view(torch.bfloat16).normal_(generator=g)
        kv_bytes = 2 * LAYERS * n * 4096 * 8 * 64 * 2
    with torch.cuda.stream(stream):
        q = torch.randn(n, LAYERS, 1024, device=dev, generator=g)
        k = torch.randn(n, LAYERS, 512, device=dev, generator=g)
        v = torch.randn(n, LAYERS, 512, device=dev, generator=g)
        out = torch.zeros(n, LAYERS, 1024, device=dev)
    stream.synchronize()
    positions = [lengths[i] - 1 for i in mine]
    pos = (C.c_int32 * n)(*positions)
    dargs = _lib.DecodeArgs(0, LAYERS, n, None, pos, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                            None, None, None, F32, F32, F32, 0, args.split)
    lib = ctx.lib

    def step(i):
        for s in range(n):
            lib.qxc_kv_set_len(arena.handle, s, positions[s])
        st = lib.qxc_decode(ctx.handle, arena.handle, C.byref(dargs))
        if st != 0:
            raise RuntimeError(lib.qxc_last_error(ctx.handle).decode())

    total, per, clk, launches = timed_steps(step, K, W, stream, timing_world, dev, local, ctx)
    my_bytes = sum(LAYERS * (2 * lengths[i] * 8 * 64 * 2 + 4 * 64 * (2 * 16 + 2 * 8)) for i in mine)
    res = {"total_ms": total, "per": per, "clocks": clk, "launches": launches, "bytes": my_bytes,
           "split": ctx.last_split, "kv_arena_bytes": kv_bytes}
    arena.close()
    ctx.close()
    return res


def config4_lengths(args):
    from qx_b200 import synthetic as syn
    return [int(x) for x in syn.uniform_int(0x51580400, 256, 128, 4096)][:args.c4_sequences]


def run_config4(args, world, rank, local):
    """Config 4: 256 independent Granite sequences, lengths U{128..4096}, bf16 KV,
    one decode step through 24 layers; sequences sharded over ranks by LPT on KV bytes."""
    from qx_b200.distributed import lpt_shard, sequence_kv_bytes
    lengths = config4_lengths(args)
    assignment, _ = lpt_shard([sequence_kv_bytes(L) for L in lengths], world)
    K, W = args.steps, args.warmup
    r = config4_measure(args, local, lengths, assignment[rank], K, W, world)
    total = r["total_ms"]
    nseq = len(lengths)
    line = base_line("multi-sequence Granite decode tok/s (256 sequences x 24 layers)", nseq * K / (total / 1e3),
                     "tok/s", world, K, W, total, True, "strong", "f32 q/k/v, bf16 KV",
                     {"workload": f"config4: {nseq} Granite sequences, lengths U{{128..4096}} (seed 0x51580400), "
                                  "24 layers, bf16 KV, one decode step each",
                      "l2": f"{r['bytes'] / 1e9:.1f} GB of KV per step",
                      "parallelism": f"sequences sharded x{world} by LPT on KV bytes, no collective"},
                     r["clocks"], r["launches"])
    line["config"]["split"] = r["split"]
    line["config"]["kv_arena_bytes_per_rank"] = int(r["kv_arena_bytes"])
    if args.paged:
        line["config"]["workload"] += f"; paged arena, {args.paged}-row pages, pool sized to the batch"
    line["roofline"] = hbm_roofline(r["bytes"], r["per"], "qx_decode_tc_kernel<bf16,TcGranitePair>",
                                    None if nseq != 256 or world != 1 else ("config4_paged" if args.paged else "config4"))
    return line


def sharded_config4(args, world, rank, local):
    """The path that shards (config 4), measured beside the config-1 headline:
    the 256 sequences split over the ranks by LPT on KV bytes, each rank
    timing its own shard (device time, max over ranks). At N > 1 rank 0 also
    times all 256 sequences alone on its GPU first (the other ranks wait), so
    the line carries the one-GPU value of the same run and the efficiency
    value / (N x one-GPU value)."""
    from qx_b200.distributed import lpt_shard, sequence_kv_bytes
    lengths = config4_lengths(args)
    K, W = args.steps, args.warmup
    one = None
    if world > 1:
        barrier(world)
        if rank == 0:
            r1 = config4_measure(args, local, lengths, list(range(len(lengths))), K, W, 1)
            one = len(lengths) * K / (r1["total_ms"] / 1e3)
        barrier(world)
    assignment, loads = lpt_shard([sequence_kv_bytes(L) for L in lengths], world)
    r = config4_measure(args, local, lengths, assignment[rank], K, W, world)
    value = len(lengths) * K / (r["total_ms"] / 1e3)
    if one is None:
        one = value
    peak, kind = hbm_peak()
    per_rank_gbs = r["bytes"] / (r["total_ms"] / K / 1e3) / 1e9
    return {"workload": f"config4: {len(lengths)} Granite sequences x 24 layers, bf16 KV, lengths U{{128..4096}} "
                        "(seed 0x51580400), sharded by LPT on KV bytes, no collective",
            "metric": "multi-sequence Granite decode tok/s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": K, "ms_per_step": r["total_ms"] / K, "scaling": "strong",
            "one_gpu_value": one, "efficiency": value / (world * one),
            "rank0_sequences": len(assignment[0]), "max_rank_kv_bytes": max(loads),
            "rank0_hbm_frac": per_rank_gbs / peak, "peak_kind": kind, "split": r["split"],
            "gpu_launches": r["launches"]}


def kv_split_config3(args, world, rank, local):
    """The path with a collective (config 3), measured beside the config-1
    headline at N > 1: one Qwen3 context of 32768 positions with its KV
    length split over the N ranks, each step's (m, l, O) partials crossing
    NVLink inside the decode grid (qxc_decode_exchange). Rank 0 first times
    the whole context alone on its GPU (the other ranks wait), so the object
    carries the one-GPU value of the same run and the speed-up."""
    import copy
    a = copy.copy(args)
    a.no_cpu_baseline = True
    a.split = 0
    a.exchange = "peer"
    # a step is ~15 us: time at least 1000 (20 graph replays), whatever the
    # headline's step count
    a.steps = max(args.steps, 1000)
    a.warmup = max(args.warmup, 100)
    one = None
    barrier(world)
    if rank == 0:
        one = run_config3(a, 1, 0, local)["value"]
    barrier(world)
    line = run_config3(a, world, rank, local)
    return {"workload": f"config3: Qwen3 layer decode, 32 q / 4 kv heads, d=128, bf16 KV, length "
                        f"{args.qwen_context}, KV length split x{world}",
            "metric": line["metric"], "value": line["value"], "unit": line["unit"], "n_gpus": world,
            "steps": line["steps"], "ms_per_step": line["ms_per_step"], "scaling": "strong",
            "one_gpu_value": one, "speedup": line["value"] / one if one else None,
            "parallelism": line["config"]["parallelism"], "split": line["config"]["split"],
            "rank0_hbm_frac": line["roofline"]["frac"], "gpu_launches": line.get("gpu_launches")}


# ---------------------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------------------
def run_reference(args, world, rank):
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import py_oracle as o
    from qx_b200 import synthetic as syn
    o.build()
    threads = os.cpu_count() or 1
    L = args.context
    if args.workload != "config1":
        return {"impl": "reference", "unavailable": f"reference arm implemented for config1 only ({args.workload})"}
    # each step: a bounded sample of the 24-layer step, `units` layers run in
    # parallel on all host threads; tok/s extrapolates to the 24 layers.
    units = max(1, min(LAYERS, threads))
    P = L - 64
    kc = syn.normal(11, (L, 8, 64))
    vc = syn.normal(12, (L, 8, 64))
    caches = []
    for _ in range(units):
        c = o.KvCache(L)
        c.keys[:], c.values[:] = kc, vc
        caches.append(c)
    qs = [syn.normal(13 + l, (1024,)) for l in range(units)]
    ks = [syn.normal(113 + l, (512,)) for l in range(units)]
    vs = [syn.normal(213 + l, (512,)) for l in range(units)]

    def step(i):
        pos = P + (i % 64)
        for c in caches:
            c.length.value = pos
        worst, _ = o.granite_decode_many(qs, ks, vs, [pos] * units, caches, threads=threads)
        assert worst == 0

    budget_steps = args.steps
    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(budget_steps):
        step(i)
        if time.perf_counter() - t0 > args.reference_budget_s:
            budget_steps = i + 1
            break
    dt = time.perf_counter() - t0
    step_s = dt / budget_steps * (LAYERS / units)
    value = 1.0 / step_s
    return {
        "impl": "reference",
        "metric": "attention-stack decode tok/s (Granite 24-layer GQA stack, batch 1 per GPU)",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": budget_steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic: seeded N(0,1)",
        "config": {"workload": f"config1: Granite-3.0-1B-A400M attention stack, 24 layers, fp32 KV, context {L}, "
                               f"positions {P}..{L - 1} cycled, batch 1", "context": L, "layers": LAYERS},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"per step {units} of the 24 layers in parallel on {threads} threads, "
                                   "extrapolated to 24 layers; oracle/qx_oracle.c restates qx-runtime "
                                   "granite_attention_decode (the Rust reference cannot be built here)"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3200)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config1",
                    choices=["config0", "config1", "config2", "config3", "config4", "layer", "commit", "verify",
                             "sweep"])
    ap.add_argument("--layer-chain", action="store_true",
                    help="layer workload: qxc_attention_layer per layer (graph-captured) instead of qxc_attention_stack")
    ap.add_argument("--no-sharded", action="store_true",
                    help="config1: leave out the `sharded` object (config 4 sharded over the ranks)")
    ap.add_argument("--no-kv-split", action="store_true",
                    help="config1 at N>1: leave out the `kv_split` object (config 3's KV length split over the ranks)")
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--split", type=int, default=0)
    ap.add_argument("--paged", type=int, default=0, help="config4: paged KV arena with this many rows per page")
    ap.add_argument("--exchange", default="peer", choices=["peer", "kernel", "nccl"],
                    help="config3 N>1: partials exchanged inside the split merge kernel (peer), by a separate "
                         "exchange kernel (kernel), or by an NCCL all-gather (nccl)")
    ap.add_argument("--prefill-len", type=int, default=2048, help="config2 prompt length (512 or 2048)")
    ap.add_argument("--qwen-context", type=int, default=32768, help="config3 KV length")
    ap.add_argument("--c4-sequences", type=int, default=256,
                    help="config4: the first N of its 256 sequences (a smaller case of the same kernel, to profile)")
    ap.add_argument("--native-exp", action="store_true", help="hardware exp2 instead of qx's pinned exp_f32")
    ap.add_argument("--e2e-steps", type=int, default=640)
    ap.add_argument("--cpu-steps", type=int, default=16)
    ap.add_argument("--reference-budget-s", type=float, default=150.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        # NCCL writes its log (its version line included, under NCCL_DEBUG)
        # to stdout unless told otherwise: keep stdout for the one JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        if args.workload == "sweep":
            # the reference's --v2-attention-sweep (tools/qx-bench/src/main.rs:8984-9080): one line per
            # context, each with its algorithmic bytes, achieved GB/s and roofline
            for L in (512, 2048, 4096):
                args.context = L
                line = run_config1(args, world, rank, local)
                line["config"]["sweep"] = [512, 2048, 4096]
                if rank == 0:
                    print(json.dumps(line), flush=True)
            return 0
        run = {"config0": run_config0, "config1": run_config1, "config2": run_config2, "config3": run_config3,
               "config4": run_config4, "layer": run_layer, "commit": run_commit,
               "verify": run_verify}[args.workload]
        line = run(args, world, rank, local)
        if args.workload == "config1" and not args.no_sharded:
            line["sharded"] = sharded_config4(args, world, rank, local)
        if args.workload == "config1" and world > 1 and not args.no_kv_split:
            try:
                line["kv_split"] = kv_split_config3(args, world, rank, local)
            except Exception as exc:  # the headline and `sharded` still print
                line["kv_split"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
