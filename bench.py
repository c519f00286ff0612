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
                    [--workload config1|config3|config4|config0]

Prints one JSON line on rank 0. N>1 runs under torchrun: one independent
sequence (replica) per GPU, no collective on the data path ("weak" scaling),
device time max-reduced over ranks. `--impl reference` times the CPU
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
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ctx.launch_count
    torch.cuda.synchronize(dev)
    barrier(world)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(K):
            ev[i][0].record(stream)
            step(i)
            ev[i][1].record(stream)
        end.record(stream)
        stream.synchronize()
    launches = ctx.launch_count - launches0
    total_ms = start.elapsed_time(end)
    kernel_ms = [a.elapsed_time(b) for a, b in ev]
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
        hq = q.cpu().numpy()
        hk = k.cpu().numpy()
        hv = v.cpu().numpy()
        hout = np.zeros((LAYERS, 1024), np.float32)
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
               "api": "qxc_decode_host (host q/k/v in, host out, synchronous)"}

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
                   "softmax_exp": "native exp2" if args.native_exp else "qx pinned exp_f32"},
        "hbm_gbs": achieved_gbs,
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                     "frac": achieved_gbs / peak, "peak_kind": peak_kind,
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
    ap.add_argument("--workload", default="config1", choices=["config1"])
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--split", type=int, default=0)
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

    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        line = run_config1(args, world, rank, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
