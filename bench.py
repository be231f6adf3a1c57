#!/usr/bin/env python
"""SKA core fwd+bwd throughput on B200 (the Koopman_Mamba SKA hot path).

Workload (one "step" = one forward + one backward of the SKA core between
the projections and eta/out_proj, over one batch of synthetic input):
    B=8 per GPU, H=12, L=2048, head dim P=64, rank r=32, chunk 64, ridge 1e-3,
    power_K=2, bf16 I/O (fp32 arithmetic); z, zq, v ~ N(0,1)/sqrt(64) and
    dy ~ N(0,1) from seed 1 (+1000*rank), one torch.Generator, in that order.
Weak scaling: every rank runs its own B=8 shard; no collective in the layer.

Prints ONE JSON line (rank 0):
  value   tokens/s over all ranks, inputs resident in HBM, device-timed with
          CUDA events per step (L2 flushed between steps, outside the events),
          max over ranks
  e2e     the same metric through the C ABI with pinned HOST buffers: each step
          copies z, zq, v, dy host->device, runs fwd+bwd, copies y, dz, dzq, dv
          back; copies inside the timed region.  `value` streams the steps with
          double-buffered device tensors (each step's copies overlap its
          neighbours' compute and copies); `serial_value` runs them one after
          another on one stream
  roofline  the dominant kernel: algorithmic bytes per launch / its average
          CUDA-event duration against MEASURED_PEAKS.json HBM bandwidth
  cpu_baseline  the numpy oracle (port of the reference's CPU path) on the
          box's host cores, N=1 only

--impl reference times the reference's CPU path (the numpy oracle port, all
host cores) on the same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

B_PER_GPU, H, L, P, R, CS, K, RIDGE = 8, 12, 2048, 64, 32, 64, 2, 1e-3
SEED = 1
METRIC = "SKA fwd+bwd tokens/sec/GPU (L=2048,r=32) and % of HBM roofline at 1/2/4/8 B200"
UNIT = "tokens/s"
WORKLOAD = "ska_core fwd+bwd B=8/GPU H=12 L=2048 P=64 r=32 chunk=64 K=2 ridge=1e-3 bf16 I/O"
L2_FLUSH_BYTES = 256 << 20   # > 126 MB L2


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-workers", type=int, default=0, help="oracle processes (0 = all cores, max 8)")
    return ap.parse_args(argv)


# ----------------------------------------------------------------------------
# CPU side: the oracle port of the reference's CPU path, in a spawn pool
# ----------------------------------------------------------------------------

def _cpu_task(args):
    """One batch element of the workload through the numpy oracle (fp32, as the
    reference computes after .float()); returns seconds."""
    (b_lo, b_hi, seed) = args
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    import numpy as np
    from oracle.ska_oracle import SkaParams, ska_core_fwd_bwd
    z, zq, v, dy = _cpu_inputs(seed)
    t0 = time.perf_counter()
    ska_core_fwd_bwd(z[b_lo:b_hi], zq[b_lo:b_hi], v[b_lo:b_hi], 1.0, dy[b_lo:b_hi],
                     SkaParams(chunk_size=CS, ridge_eps=RIDGE, power_K=K), np.float32)
    return time.perf_counter() - t0


_CPU_CACHE = {}


def _cpu_inputs(seed):
    if seed not in _CPU_CACHE:
        import torch
        g = torch.Generator().manual_seed(seed)
        s = 1.0 / math.sqrt(64)
        z = torch.randn(B_PER_GPU, L, H, R, generator=g) * s
        zq = torch.randn(B_PER_GPU, L, H, R, generator=g) * s
        v = torch.randn(B_PER_GPU, L, H, P, generator=g) * s
        dy = torch.randn(B_PER_GPU, L, H, P, generator=g)
        _CPU_CACHE[seed] = [t.bfloat16().float().numpy() for t in (z, zq, v, dy)]
    return _CPU_CACHE[seed]


def _make_pool(workers):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    env_threads = {"OMP_NUM_THREADS": "1", "OPENBLAS_NUM_THREADS": "1", "MKL_NUM_THREADS": "1"}
    os.environ.update(env_threads)
    return ctx.Pool(workers)


def cpu_step(pool, workers):
    """One step of the CPU path: the full B=8 batch split over the workers; the
    step time is the wall time of the parallel map."""
    tasks = [(b, b + 1, SEED) for b in range(B_PER_GPU)]
    t0 = time.perf_counter()
    pool.map(_cpu_task, tasks, chunksize=1)
    return time.perf_counter() - t0


def cpu_workers(n):
    cores = os.cpu_count() or 1
    return max(1, min(B_PER_GPU, cores if n <= 0 else n))


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    workers = cpu_workers(args.cpu_workers)
    pool = _make_pool(workers)
    try:
        pool.map(_cpu_inputs_warm, [SEED] * workers)
        for _ in range(max(args.warmup, 1)):
            cpu_step(pool, workers)
        times = [cpu_step(pool, workers) for _ in range(args.steps)]
    finally:
        pool.close()
        pool.join()
    total = sum(times)
    value = B_PER_GPU * L * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "compute": "numpy fp32 on the host cores (the reference's fp32 upcast of the bf16 tensors)",
        "data": "synthetic (seeded N(0,1)/8 inputs, bf16-rounded)",
        "config": {"workload": WORKLOAD, "path": "reference CPU path: numpy oracle port of "
                   "koopman_lm/ska.py (PyTorch backend) fwd+bwd, fp32", "io_dtype": "bf16-rounded"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": workers, "kind": "port",
                         "sample": f"full B=8 batch per step, one batch element per process"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _cpu_inputs_warm(seed):
    _cpu_inputs(seed)
    return 0


# ----------------------------------------------------------------------------
# GPU side
# ----------------------------------------------------------------------------

class ClockSampler:
    """SM clock, power and clock-event reasons sampled by NVML every 2 ms in a
    background thread; `stop` keeps the samples taken inside [t0, t1] (the timed
    region), or all of them when that window is shorter than the sampling period."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self):
        self.thread = None
        self.samples = []
        self.handle = None

    def start(self, device_index):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = self._handle(pynvml, device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None
            return
        self.stop_flag = threading.Event()

        def run():
            nv, h = self.nvml, self.handle
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self.stop_flag.is_set():
                try:
                    self.samples.append((time.perf_counter(), nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                         get_reasons(h), nv.nvmlDeviceGetPowerUsage(h) / 1000.0))
                except Exception:
                    pass
                time.sleep(0.002)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        time.sleep(0.02)   # first samples before the timed region

    @staticmethod
    def _handle(nv, device_index):
        import torch
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            return nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            ids = [int(x) for x in vis.split(",") if x.strip().isdigit()]
            return nv.nvmlDeviceGetHandleByIndex(ids[device_index] if ids else device_index)

    def stop(self, t0, t1):
        if self.thread is None:
            return None
        time.sleep(0.01)
        self.stop_flag.set()
        self.thread.join(timeout=2)
        inside = [x for x in self.samples if t0 <= x[0] <= t1]
        use = inside if len(inside) >= 3 else self.samples
        if not use:
            return None
        reasons = sorted({n for _, _, bits, _ in use for n, b in self.REASONS if bits & b})
        return {"sm_mhz": statistics.median(x[1] for x in use), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "power_w_max": max(x[3] for x in use), "samples": len(use),
                "window": "timed region" if use is inside else "warm-up + timed region (timed region < 3 samples)"}


def _visible_gpu_indices(world, local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [int(x) for x in vis.split(",") if x.strip().isdigit()]
        return ids[:max(world, 1)] if ids else None
    return list(range(max(world, 1)))


def _measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _ncu_traffic():
    """Per-launch DRAM traffic of each kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return {}


# Bytes each kernel must move per launch (bf16 token tensors, fp32 chunk records):
# its token-tensor reads and writes plus the per-chunk records it reads or
# writes, each once.  C = chunks per series; SW = floats per statistics record.
def _kernel_algo_bytes(tokens_heads):
    es = 2
    chunks = tokens_heads // CS
    rec = (2 * R * R + P * R) * 4          # one statistics record
    wrec = P * R * 4                       # dW' record / W planes
    return {
        "k_fwd_stats": tokens_heads * (R + P) * es + chunks * rec,          # z, v -> records
        "k_stats_scan": tokens_heads * (R + P) * es + chunks * rec,         # z, v -> scanned records
        "k_scan_fwd": 2 * chunks * rec,                                      # records in place
        "k_fwd_chunk": tokens_heads * (R + P) * es + chunks * rec,          # records, zq -> y
        "k_dw": tokens_heads * (R + P) * es + chunks * wrec,                # zq, dy -> dW'
        "k_bwd_chunk": chunks * (2 * rec + 2 * wrec),                        # records, dW' -> d records, W
        "k_scan_bwd": 2 * chunks * rec,                                      # d records in place
        "k_bwd_tok": tokens_heads * (R + 2 * P + 2 * R + P) * es + chunks * (rec + wrec),
        # z, v, dy, d records, W -> dz, dzq, dv
    }


KERNELS = ("k_fwd_stats", "k_scan_fwd", "k_fwd_chunk", "k_dw", "k_bwd_chunk", "k_scan_bwd", "k_bwd_tok")


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference_arm(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    want_cpu = (not args.no_cpu_baseline) and world == 1 and rank == 0
    pool = None
    workers = cpu_workers(args.cpu_workers)
    if want_cpu:
        pool = _make_pool(workers)   # spawn pool started before any CUDA work

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from koopman_mamba_b200 import _lib
    from koopman_mamba_b200.sharding import max_over_ranks

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- inputs (generated on the host from the seed, moved to HBM untimed) ----
    g = torch.Generator().manual_seed(SEED + 1000 * rank)
    s = 1.0 / math.sqrt(64)
    host = [torch.randn(B_PER_GPU, L, H, n, generator=g) * s for n in (R, R, P)]
    host.append(torch.randn(B_PER_GPU, L, H, P, generator=g))
    host = [t.bfloat16().pin_memory() for t in host]
    z, zq, v, dy = (t.to(dev) for t in host)
    y = torch.empty(B_PER_GPU, L, H, P, dtype=torch.bfloat16, device=dev)
    dz, dzq, dv = torch.empty_like(z), torch.empty_like(zq), torch.empty_like(v)
    gamma = torch.ones((), dtype=torch.float32, device=dev)
    dgamma = torch.empty((), dtype=torch.float32, device=dev)
    shape = _lib.make_shape(B_PER_GPU, L, H, R, P, CS, K, RIDGE)
    saved_bytes, scratch_bytes = _lib.workspace_size(shape)
    saved = torch.empty(saved_bytes, dtype=torch.uint8, device=dev)
    scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)

    def desc(t):
        return _lib.SkaTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))

    D = {n: desc(t) for n, t in dict(z=z, zq=zq, v=v, dy=dy, y=y, dz=dz, dzq=dzq, dv=dv).items()}
    BF16 = _lib.SKA_DTYPE_BF16
    gp, dgp = ctypes.c_void_p(gamma.data_ptr()), ctypes.c_void_p(dgamma.data_ptr())
    savp, scrp = ctypes.c_void_p(saved.data_ptr()), ctypes.c_void_p(scratch.data_ptr())
    byref = ctypes.byref

    def step(Dx=D):
        rc = lib.ska_fwd(byref(shape), BF16, byref(Dx["z"]), byref(Dx["zq"]), byref(Dx["v"]), gp, byref(Dx["y"]),
                         savp, saved_bytes, sp)
        if rc:
            _lib.check("ska_fwd", rc)
        rc = lib.ska_bwd(byref(shape), BF16, byref(Dx["z"]), byref(Dx["zq"]), byref(Dx["v"]), gp, byref(Dx["dy"]),
                         savp, saved_bytes, scrp, scratch_bytes, byref(Dx["dz"]), byref(Dx["dzq"]),
                         byref(Dx["dv"]), dgp, sp)
        if rc:
            _lib.check("ska_bwd", rc)

    # per-kernel events (recorded by the library on the launch stream)
    kev = [torch.cuda.Event(enable_timing=True) for _ in range(_lib.SKA_PROFILE_EVENTS)]
    for e in kev:
        e.record(stream)
    handles = (ctypes.c_void_p * len(kev))(*[e.cuda_event for e in kev])
    _lib.check("ska_set_profile_events", lib.ska_set_profile_events(handles, len(kev)))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps, device-timed per step, L2 flushed in between ----
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # statistics and scan are one kernel where the layout takes the fused path
    fused_scan = lib.ska_kernel_path(byref(shape), BF16, byref(D["z"]), byref(D["v"])) & _lib.SKA_PATH_FUSED_SCAN
    names = ("k_stats_scan",) + KERNELS[2:] if fused_scan else KERNELS
    # profile-event pairs bounding each forward kernel
    fwd_pairs = ((0, 2), (2, 3)) if fused_scan else ((0, 1), (1, 2), (2, 3))
    per_kernel = {k: [] for k in names}
    clocks = ClockSampler()
    clocks.start(local)
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.zero_()
        ev0[i].record(stream)
        step()
        ev1[i].record(stream)
        kev[-1].synchronize()
        spans = [kev[a].elapsed_time(kev[b]) for a, b in fwd_pairs] + \
                [kev[j].elapsed_time(kev[j + 1]) for j in (4, 5, 6, 7)]
        for k, ms in zip(names, spans):
            per_kernel[k].append(ms)
    torch.cuda.synchronize()
    barrier()
    wall1 = time.perf_counter()
    wall = wall1 - wall0
    clock_info = clocks.stop(wall0, wall1)
    dev_ms = sum(a.elapsed_time(b) for a, b in zip(ev0, ev1))
    dev_ms_max = max_over_ranks(dev_ms, dev)
    tokens_per_step = world * B_PER_GPU * L
    value = tokens_per_step * args.steps / (dev_ms_max / 1e3)

    # ---- end to end through the C ABI with host buffers ----
    e2e = None
    if not args.no_e2e:
        out_host = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (y, dz, dzq, dv)]
        h2d = sum(t.numel() * t.element_size() for t in host)
        d2h = sum(t.numel() * t.element_size() for t in out_host)
        ea = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        eb = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]

        def e2e_step():
            for src, dst in zip(host, (z, zq, v, dy)):
                dst.copy_(src, non_blocking=True)
            step()
            for src, dst in zip((y, dz, dzq, dv), out_host):
                dst.copy_(src, non_blocking=True)

        for _ in range(max(1, args.warmup // 2)):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        for i in range(args.steps):
            ea[i].record(stream)
            e2e_step()
            eb[i].record(stream)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(ea, eb)), dev)
        serial = tokens_per_step * args.steps / (e_ms / 1e3)

        # The same steps as a stream of batches: two device buffer sets; step i copies its
        # inputs host->device on one stream and its results device->host on another,
        # overlapping step i - 1's compute and copies (the link is full duplex).  Every
        # step's copies stay inside the timed region, which spans all K steps.
        din = [(z, zq, v, dy), tuple(torch.empty_like(t) for t in (z, zq, v, dy))]
        dout = [(y, dz, dzq, dv), tuple(torch.empty_like(t) for t in (y, dz, dzq, dv))]
        Dset = [{n: desc(t) for n, t in zip(("z", "zq", "v", "dy", "y", "dz", "dzq", "dv"), din[k] + dout[k])}
                for k in range(2)]
        outs = [out_host, [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (y, dz, dzq, dv)]]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in, ev_comp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

        def piped_step(i):
            k = i % 2
            s_in.wait_event(ev_comp[k])          # step i - 2's compute has read this input set
            with torch.cuda.stream(s_in):
                for src, dst in zip(host, din[k]):
                    dst.copy_(src, non_blocking=True)
            ev_in[k].record(s_in)
            stream.wait_event(ev_in[k])
            stream.wait_event(ev_out[k])         # step i - 2's results have left this output set
            step(Dset[k])
            ev_comp[k].record(stream)
            s_out.wait_event(ev_comp[k])
            with torch.cuda.stream(s_out):
                for src, dst in zip(dout[k], outs[k]):
                    dst.copy_(src, non_blocking=True)
            ev_out[k].record(s_out)

        for i in range(2):
            piped_step(i)
        torch.cuda.synchronize()
        barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        s_in.wait_event(p0)
        for i in range(args.steps):
            piped_step(i)
        for k in range(2):
            stream.wait_event(ev_out[k])
        p1.record(stream)
        torch.cuda.synchronize()
        p_ms = max_over_ranks(p0.elapsed_time(p1), dev)
        e2e = {"value": tokens_per_step * args.steps / (p_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "copies": "double-buffered: host->device and device->host on two copy streams, overlapping "
                         "the neighbouring steps' compute and copies",
               "serial_value": serial}

    lib.ska_set_profile_events(None, 0)
    # stats (+ scan), chunk operators; dW', chunk backward, scan, token backward
    launches_per_step = 6 if fused_scan else 7

    # ---- roofline of the dominant kernel ----
    peak, peak_kind = _measured_peaks()
    algo = _kernel_algo_bytes(B_PER_GPU * L * H)
    avg_ms = {k: statistics.mean(vv) for k, vv in per_kernel.items()}
    dom = max(avg_ms, key=avg_ms.get)
    ach = algo[dom] / (avg_ms[dom] / 1e3) / 1e9
    traffic = _ncu_traffic().get(dom)
    # the step's unique token traffic: forward z, zq, v -> y (2r + 2P); backward z, zq, v, dy -> dz, dzq,
    # dv (2r + 2P read, 2r + P written): (6r + 5P) bf16 values per token and head
    step_algo = B_PER_GPU * L * H * (6 * R + 5 * P) * 2
    roofline = {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": peak, "unit": "GB/s",
                "frac": ach / peak, "traffic": traffic, "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                "algo_bytes_per_launch": algo[dom],
                "step": {"algo_bytes": step_algo, "achieved": step_algo / (dev_ms / args.steps / 1e3) / 1e9,
                         "frac": step_algo / (dev_ms / args.steps / 1e3) / 1e9 / peak},
                "kernels_ms": {k: round(vv, 4) for k, vv in avg_ms.items()}}

    cpu = None
    if want_cpu:
        try:
            pool.map(_cpu_inputs_warm, [SEED] * workers)
            cpu_step(pool, workers)
            ts = [cpu_step(pool, workers) for _ in range(2)]
            cpu = {"value": B_PER_GPU * L / min(ts), "unit": UNIT, "cores": workers, "kind": "port",
                   "sample": "full B=8 batch (16384 tokens x 12 heads), numpy oracle fp32, best of 2 after 1 warm-up"}
        finally:
            pool.close()
            pool.join()

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "compute": "bf16 token tensors; token-level tcgen05 products (fp32 operands as bf16 hi+lo "
                       "pairs); chunk algebra as 3-term-split TF32 mma.sync (fp32-level); fp32 accumulation, "
                       "Cholesky, inverse and power iteration",
            "data": "synthetic (seeded N(0,1)/8 inputs, N(0,1) upstream grad)",
            "config": {"workload": WORKLOAD, "B_per_gpu": B_PER_GPU, "H": H, "L": L, "P": P, "r": R, "chunk": CS,
                       "power_K": K, "io_dtype": "bf16", "parallelism": f"dp{world} (batch shards, no collective)",
                       "l2": "flushed between timed steps (256 MiB write outside the events); working set > L2"},
            "e2e": e2e, "gpu_launches": launches_per_step * args.steps, "roofline": roofline,
            "cpu_baseline": cpu, "clocks": clock_info, "wall_s": wall,
        }
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
