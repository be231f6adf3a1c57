#!/usr/bin/env python
"""SKA core throughput on B200 (the Koopman_Mamba Spectral Koopman Attention hot path).

Two workloads, both synthetic with the reference configurations' shapes:
  c2 (headline)  forward + backward, B=8 per GPU, H=12, L=2048, head dim P=64,
                 rank r=32, chunk 64, ridge 1e-3, power_K=2, bf16 I/O (fp32
                 arithmetic); z, zq, v ~ N(0,1)/sqrt(64) and dy ~ N(0,1) from seed
                 1 (+1000*rank), one torch.Generator, in that order.  Weak
                 scaling: every rank runs its own B=8 batch; no collective.
  c3             long-context forward, B=1, H=16, L=32768, P=64, r=64, chunk 128,
                 bf16 I/O; z, zq, v ~ N(0,1)/sqrt(64) from seed 2.  Strong
                 scaling: the 16 heads are split over the ranks (contiguous head
                 shards); no collective.
A "step" is one pass of the SKA core (c2: forward + backward, c3: forward) over
one batch, between the projections and eta/out_proj, through the C ABI.

The default run prints ONE JSON line (rank 0) for c2 and carries the c3
measurement of the same run (same ranks) as its "c3" object; --workload c3 prints
the c3 line alone.  Fields:
  value     tokens/s of the whole job, inputs resident in HBM, device-timed with
            CUDA events around each of the K steps (L2 flushed between steps by a
            256 MiB write outside the events; no host synchronisation inside the
            timed region), max over ranks
  e2e       the same metric through the C ABI with pinned HOST buffers: every step
            copies its inputs host->device and its outputs device->host inside
            the timed region (double-buffered: copies of neighbouring steps overlap
            on two copy streams; `serial_value`: one stream, one step at a time);
            per-rank copy bandwidth in GB/s
  roofline  the step's algorithmic token bytes (bf16; c2 2*(6r+5P), c3 2*(2r+2P)
            per token and head) / step time, against MEASURED_PEAKS.json hbm_gbs;
            `kernels` gives each kernel's share from a separate per-kernel event
            pass, and `traffic` the DRAM bytes per step from the committed ncu
            capture (profiles/ncu_traffic.json) with its ratio to the algorithmic
            bytes
  sustained ~1 s of back-to-back steps after the timed region with NVML clocks
            (the K-step timed region is short; this shows the clocks under load)
  cpu_baseline  the reference's CPU path restated in PyTorch (oracle/ska_torch_port.py,
            which runs at the reference's own CPU speed) on the box's host cores,
            rank 0 at N=1 only, best of 3 after 1 warm-up

--impl reference times that same CPU path (all host cores, one series slice per
process) on the same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "SKA fwd+bwd tokens/sec/GPU (L=2048,r=32) and % of HBM roofline at 1/2/4/8 B200"
METRIC_C3 = "SKA fwd tokens/s, long context (L=32768, r=64), heads split over the GPUs"
METRICS = {"c2": METRIC, "c3": METRIC_C3,
           "c4": "SKA fwd+bwd tokens/sec/GPU, the 50M hybrid LM's SKA layer (H=7, r=48)",
           "c5": "SKA fwd tokens/sec/GPU, the 2-layer recall model's SKA layer (H=4, r=16, P=32)"}
UNIT = "tokens/s"
L2_FLUSH_BYTES = 256 << 20   # > 126 MB L2

WORKLOADS = {
    "c2": dict(B=8, H=12, L=2048, P=64, r=32, CS=64, K=2, ridge=1e-3, seed=1, bwd=True, scaling="weak",
               name="ska_core fwd+bwd B=8/GPU H=12 L=2048 P=64 r=32 chunk=64 K=2 ridge=1e-3 bf16 I/O"),
    "c3": dict(B=1, H=16, L=32768, P=64, r=64, CS=128, K=2, ridge=1e-3, seed=2, bwd=False, scaling="strong",
               name="ska_core fwd B=1 H=16 (heads split over the GPUs) L=32768 P=64 r=64 chunk=128 K=2 "
                    "ridge=1e-3 bf16 I/O"),
    # the SKA layers of the two model configurations, as core workloads of their own
    "c4": dict(B=32, H=7, L=2048, P=64, r=48, CS=64, K=2, ridge=1e-3, seed=3, bwd=True, scaling="weak",
               name="ska_core fwd+bwd, the SKA layer of the 50M hybrid LM: B=32/GPU H=7 L=2048 P=64 r=48 "
                    "chunk=64 K=2 ridge=1e-3 bf16 I/O"),
    "c5": dict(B=256, H=4, L=1024, P=32, r=16, CS=64, K=2, ridge=1e-3, seed=4, bwd=False, scaling="weak",
               name="ska_core fwd, the SKA layer of the 2-layer recall model: B=256/GPU H=4 L=1024 P=32 r=16 "
                    "chunk=64 K=2 ridge=1e-3 bf16 I/O"),
}


LM_WORKLOAD = ("hybrid Mamba-2 + SKA LM training step: config_50m_mamba_attn hyper-parameters with its attention "
               "layers [2, 5, 8] as SKA layers (d_model 448, 12 layers, SKA H=7 r=48 P=64, d_state 128, vocab 32000), "
               "batch 32 x 2048 tokens per GPU, bf16 autocast, AdamW, DDP with an NCCL gradient all-reduce")


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("c2", "c3", "c4", "c5", "lm"), default="c2",
                    help="c2 (default, with a c3 block), c3, c4, c5, or lm (the 50M hybrid model's training step)")
    ap.add_argument("--no-c3", action="store_true", help="skip the c3 block of the default c2 run")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sustained", action="store_true")
    ap.add_argument("--cpu-workers", type=int, default=0, help="oracle processes (0 = all cores, max 8)")
    return ap.parse_args(argv)


def algo_bytes_per_token_head(wl):
    """Unique bf16 token bytes per token and head (forward: z, zq, v in, y out;
    backward: z, zq, v, dy in, dz, dzq, dv out)."""
    r, P = wl["r"], wl["P"]
    return 2 * ((6 * r + 5 * P) if wl["bwd"] else (2 * r + 2 * P))


def head_range(wl, world, rank):
    """Heads of this rank: all of them for weak scaling, a contiguous share otherwise."""
    from koopman_mamba_b200.sharding import shard_range
    if wl["scaling"] == "weak":
        return 0, wl["H"]
    return shard_range(wl["H"], world, rank)


def rank_seed(wl, rank):
    return wl["seed"] + (1000 * rank if wl["scaling"] == "weak" else 0)


def host_inputs(wl, rank, world, dy=True):
    """This rank's z, zq, v (and dy) as float32 CPU tensors, bf16-rounded."""
    import torch
    g = torch.Generator().manual_seed(rank_seed(wl, rank))
    s = 1.0 / math.sqrt(64)
    B, L, H = wl["B"], wl["L"], wl["H"]
    out = [torch.randn(B, L, H, n, generator=g) * s for n in (wl["r"], wl["r"], wl["P"])]
    if dy and wl["bwd"]:
        out.append(torch.randn(B, L, H, wl["P"], generator=g))
    lo, hi = head_range(wl, world, rank)
    return [t[:, :, lo:hi].contiguous().bfloat16().float() for t in out]


# ----------------------------------------------------------------------------
# CPU side: the PyTorch restatement of the reference's CPU path, in a spawn pool
# ----------------------------------------------------------------------------

_CPU_CACHE = {}


def _cpu_inputs(key):
    if key not in _CPU_CACHE:
        wl = WORKLOADS[key]
        _CPU_CACHE[key] = host_inputs(wl, 0, 1)
    return _CPU_CACHE[key]


def _cpu_task(args):
    """One slice of the workload through the PyTorch CPU restatement of the
    reference's path (fp32 after the bf16 rounding, as the reference computes after
    .float(); autograd backward), one thread; returns seconds."""
    key, b, h_lo, h_hi = args
    import torch
    from oracle.ska_torch_port import ska_core_torch
    torch.set_num_threads(1)
    wl = WORKLOADS[key]
    x = [a[b:b + 1, :, h_lo:h_hi].contiguous() for a in _cpu_inputs(key)]
    t0 = time.perf_counter()
    if wl["bwd"]:
        z, zq, v = (t.clone().requires_grad_(True) for t in x[:3])
        g = torch.tensor(1.0, requires_grad=True)
        ska_core_torch(z, zq, v, g, chunk_size=wl["CS"], ridge_eps=wl["ridge"], power_K=wl["K"]).backward(x[3])
    else:
        with torch.no_grad():
            ska_core_torch(x[0], x[1], x[2], torch.tensor(1.0), chunk_size=wl["CS"], ridge_eps=wl["ridge"],
                           power_K=wl["K"])
    return time.perf_counter() - t0


def _cpu_warm(key):
    _cpu_inputs(key)
    return 0


def _make_pool(workers):
    import multiprocessing as mp
    os.environ.update({"OMP_NUM_THREADS": "1", "OPENBLAS_NUM_THREADS": "1", "MKL_NUM_THREADS": "1"})
    return mp.get_context("spawn").Pool(workers)


def cpu_tasks(key):
    """The whole workload as independent series slices: fwd+bwd workloads one batch
    element per task, forward-only ones one (batch element, head) per task."""
    wl = WORKLOADS[key]
    if wl["bwd"]:
        return [(key, b, 0, wl["H"]) for b in range(wl["B"])]
    return [(key, b, h, h + 1) for b in range(wl["B"]) for h in range(wl["H"])]


def cpu_step(pool, key):
    t0 = time.perf_counter()
    pool.map(_cpu_task, cpu_tasks(key), chunksize=1)
    return time.perf_counter() - t0


def cpu_workers(n):
    cores = os.cpu_count() or 1
    return max(1, min(8, cores if n <= 0 else n))


def cpu_baseline(pool, workers, key, repeats=3):
    wl = WORKLOADS[key]
    pool.map(_cpu_warm, [key] * workers)
    cpu_step(pool, key)
    ts = [cpu_step(pool, key) for _ in range(repeats)]
    what = "fwd+bwd" if wl["bwd"] else "fwd"
    return {"value": wl["B"] * wl["L"] / min(ts), "unit": UNIT, "cores": workers, "kind": "port",
            "sample": f"the whole {key} workload ({wl['B']}x{wl['L']} tokens x {wl['H']} heads, {what}), PyTorch "
                      f"CPU restatement of the reference path (fp32, autograd backward), {len(cpu_tasks(key))} "
                      f"series slices over {workers} single-thread processes, best of {repeats} after 1 warm-up",
            "seconds": [round(t, 4) for t in ts]}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    key = args.workload
    wl = WORKLOADS[key]
    workers = cpu_workers(args.cpu_workers)
    pool = _make_pool(workers)
    try:
        pool.map(_cpu_warm, [key] * workers)
        for _ in range(max(args.warmup, 1)):
            cpu_step(pool, key)
        times = [cpu_step(pool, key) for _ in range(args.steps)]
    finally:
        pool.close()
        pool.join()
    total = sum(times)
    value = wl["B"] * wl["L"] * args.steps / total
    line = {
        "impl": "reference", "metric": METRICS[key], "value": value, "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": wl["scaling"], "vs_baseline": None, "dtype": "f32",
        "compute": "PyTorch fp32 on the host cores (the reference's fp32 upcast of the bf16 tensors; batched "
                   "LAPACK Cholesky and solves, autograd backward)",
        "data": "synthetic (seeded N(0,1)/8 inputs, bf16-rounded)",
        "config": {"workload": wl["name"], "path": "reference CPU path: PyTorch restatement of "
                   "koopman_lm/ska.py (PyTorch backend), fp32", "io_dtype": "bf16-rounded"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": workers, "kind": "port",
                         "sample": f"the whole workload per step, {len(cpu_tasks(key))} series slices over "
                                   f"{workers} processes"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# GPU side
# ----------------------------------------------------------------------------

class ClockSampler:
    """SM clock, power and clock-event reasons sampled by NVML every 2 ms in a
    background thread; `stop` keeps the samples taken inside [t0, t1]."""

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
        time.sleep(0.02)

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


def _measured_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _ncu_traffic(key, names):
    """DRAM bytes per step (read + write of every kernel of the step) from the
    committed ncu capture of the same kernels, or None when the capture does not
    cover the kernels this library launches."""
    try:
        with open(os.path.join(REPO, "profiles", "ncu_traffic.json")) as f:
            per = json.load(f)[key]["bytes_per_launch"]
    except Exception:
        return None
    if any(n not in per for n in names):
        return None
    return sum(per[n] for n in names)


class Runner:
    """One rank's share of a workload: device tensors, caller-owned workspace and the
    C-ABI calls of one step."""

    def __init__(self, key, rank, world, dev, lib, _lib):
        import torch
        self.key, self.wl = key, WORKLOADS[key]
        wl = self.wl
        self.dev, self.lib, self.L = dev, lib, _lib
        self.h_lo, self.h_hi = head_range(wl, world, rank)
        self.H = self.h_hi - self.h_lo
        self.host = [t.bfloat16().pin_memory() for t in host_inputs(wl, rank, world)]
        self.din = [t.to(dev) for t in self.host]
        B, Lq, H, P = wl["B"], wl["L"], self.H, wl["P"]
        bf = torch.bfloat16
        self.dout = [torch.empty(B, Lq, H, P, dtype=bf, device=dev)]
        if wl["bwd"]:
            self.dout += [torch.empty_like(self.din[0]), torch.empty_like(self.din[1]), torch.empty_like(self.din[2])]
        self.gamma = torch.ones((), dtype=torch.float32, device=dev)
        self.dgamma = torch.empty((), dtype=torch.float32, device=dev)
        self.shape = _lib.make_shape(B, Lq, H, wl["r"], P, wl["CS"], wl["K"], wl["ridge"])
        self.saved_bytes, self.scratch_bytes = _lib.workspace_size(self.shape)
        if not wl["bwd"]:   # no backward reads the buffer: the forward keeps no chunk operators
            self.saved_bytes = _lib.forward_workspace_size(self.shape)
        self.saved = torch.empty(self.saved_bytes, dtype=torch.uint8, device=dev)
        self.scratch = torch.empty(self.scratch_bytes if wl["bwd"] else 256, dtype=torch.uint8, device=dev)
        self.stream = torch.cuda.current_stream(dev)
        self.sp = ctypes.c_void_p(self.stream.cuda_stream)
        self.tokens = B * Lq                   # tokens of this rank's step (each with H heads)
        self.token_heads = B * Lq * H
        self.D = self.descs(self.din, self.dout)
        self.path = lib.ska_kernel_path(ctypes.byref(self.shape), _lib.SKA_DTYPE_BF16, ctypes.byref(self.D["z"]),
                                        ctypes.byref(self.D["v"]))

    def descs(self, din, dout):
        names_in = ("z", "zq", "v", "dy")[:len(din)]
        names_out = ("y", "dz", "dzq", "dv")[:len(dout)]
        return {n: self.L.SkaTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))
                for n, t in list(zip(names_in, din)) + list(zip(names_out, dout))}

    def step(self, D=None):
        D = D or self.D
        L, lib, byref = self.L, self.lib, ctypes.byref
        gp = ctypes.c_void_p(self.gamma.data_ptr())
        savp = ctypes.c_void_p(self.saved.data_ptr())
        rc = lib.ska_fwd(byref(self.shape), L.SKA_DTYPE_BF16, byref(D["z"]), byref(D["zq"]), byref(D["v"]), gp,
                         byref(D["y"]), savp, self.saved_bytes, self.sp)
        if rc:
            L.check("ska_fwd", rc)
        if self.wl["bwd"]:
            rc = lib.ska_bwd(byref(self.shape), L.SKA_DTYPE_BF16, byref(D["z"]), byref(D["zq"]), byref(D["v"]), gp,
                             byref(D["dy"]), savp, self.saved_bytes, ctypes.c_void_p(self.scratch.data_ptr()),
                             self.scratch_bytes, byref(D["dz"]), byref(D["dzq"]), byref(D["dv"]),
                             ctypes.c_void_p(self.dgamma.data_ptr()), self.sp)
            if rc:
                L.check("ska_bwd", rc)

    def kernel_names(self):
        """The kernels one step launches, in order (from the layout's path bits)."""
        L, p = self.L, self.path
        names = ["k_stats_scan"] if p & L.SKA_PATH_FUSED_SCAN else ["k_fwd_stats", "k_scan_fwd"]
        names.append("k_fwd_chunk")
        if p & L.SKA_PATH_TC_READOUT_FWD:
            names.append("k_readout")
        if self.wl["bwd"]:
            full = bool(p & L.SKA_PATH_TC_READOUT_BWD)
            names += (["k_dw"] if full else []) + ["k_bwd_chunk", "k_scan_bwd", "k_bwd_tok"]
        return names

    def check_status(self):
        bad, code = ctypes.c_int64(0), ctypes.c_int(0)
        rc = self.lib.ska_check_status(ctypes.byref(self.shape), ctypes.c_void_p(self.saved.data_ptr()),
                                       self.saved_bytes,
                                       ctypes.c_void_p(self.scratch.data_ptr()) if self.wl["bwd"] else None,
                                       self.scratch_bytes, self.sp, ctypes.byref(bad), ctypes.byref(code))
        self.L.check("ska_check_status", rc)


def timed_steps(run, steps, flush, barrier):
    """K steps, each bracketed by CUDA events on the launching stream, the L2 flush
    between them outside the events; no host synchronisation until the end."""
    import torch
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        flush.zero_()
        ev0[i].record(run.stream)
        run.step()
        ev1[i].record(run.stream)
    torch.cuda.synchronize()
    barrier()
    t1 = time.perf_counter()
    return sum(a.elapsed_time(b) for a, b in zip(ev0, ev1)), t0, t1


def per_kernel_ms(run, n, flush):
    """Average duration of each kernel of a step, from the library's profile events
    (a separate pass after the timed region, host-synchronised per step)."""
    import torch
    lib, L = run.lib, run.L
    kev = [torch.cuda.Event(enable_timing=True) for _ in range(L.SKA_PROFILE_EVENTS)]
    for e in kev:
        e.record(run.stream)
    handles = (ctypes.c_void_p * len(kev))(*[e.cuda_event for e in kev])
    L.check("ska_set_profile_events", lib.ska_set_profile_events(handles, len(kev)))
    names = run.kernel_names()
    fused = bool(run.path & L.SKA_PATH_FUSED_SCAN)
    fwd_pairs = [(0, 2), (2, 3)] if fused else [(0, 1), (1, 2), (2, 3)]
    if "k_readout" in names:
        fwd_pairs.append((3, 9))
    bwd_pairs = []
    if run.wl["bwd"]:
        bwd_pairs = ([(4, 5)] if "k_dw" in names else []) + [(5, 6), (6, 7), (7, 8)]
    acc = {k: [] for k in names}
    try:
        for _ in range(n):
            flush.zero_()
            run.step()
            kev[8 if run.wl["bwd"] else 9].synchronize()
            spans = [kev[a].elapsed_time(kev[b]) for a, b in fwd_pairs + bwd_pairs]
            for k, ms in zip(names, spans):
                acc[k].append(ms)
    finally:
        lib.ska_set_profile_events(None, 0)
    return {k: statistics.mean(v) for k, v in acc.items()}


def e2e_measure(run, steps, warmup, barrier, max_over_ranks):
    """Through the C ABI with pinned host buffers, copies inside the timed region."""
    import torch
    dev, stream = run.dev, run.stream
    host_out = [[torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in run.dout] for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in run.host)
    d2h = sum(t.numel() * t.element_size() for t in run.dout)

    def serial_step():
        for src, dst in zip(run.host, run.din):
            dst.copy_(src, non_blocking=True)
        run.step()
        for src, dst in zip(run.dout, host_out[0]):
            dst.copy_(src, non_blocking=True)

    for _ in range(max(1, warmup // 2)):
        serial_step()
    torch.cuda.synchronize()
    barrier()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for _ in range(steps):
        serial_step()
    eb.record(stream)
    torch.cuda.synchronize()
    serial_ms = max_over_ranks(ea.elapsed_time(eb), dev)

    # copy bandwidth of this rank alone (host->device, device->host), one direction at a time
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for src, dst in zip(run.host, run.din):
        dst.copy_(src, non_blocking=True)
    c1.record(stream)
    c2, c3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c2.record(stream)
    for src, dst in zip(run.dout, host_out[0]):
        dst.copy_(src, non_blocking=True)
    c3.record(stream)
    torch.cuda.synchronize()
    h2d_gbs = h2d / (c0.elapsed_time(c1) / 1e3) / 1e9
    d2h_gbs = d2h / (c2.elapsed_time(c3) / 1e3) / 1e9

    # pipelined: two device buffer sets; step i's inputs go in on one copy stream and
    # its results out on another, overlapping steps i-1 and i+1
    din = [run.din, [torch.empty_like(t) for t in run.din]]
    dout = [run.dout, [torch.empty_like(t) for t in run.dout]]
    Dset = [run.descs(din[k], dout[k]) for k in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in, ev_comp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

    def piped_step(i):
        k = i % 2
        s_in.wait_event(ev_comp[k])
        with torch.cuda.stream(s_in):
            for src, dst in zip(run.host, din[k]):
                dst.copy_(src, non_blocking=True)
        ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        stream.wait_event(ev_out[k])
        run.step(Dset[k])
        ev_comp[k].record(stream)
        s_out.wait_event(ev_comp[k])
        with torch.cuda.stream(s_out):
            for src, dst in zip(dout[k], host_out[k]):
                dst.copy_(src, non_blocking=True)
        ev_out[k].record(s_out)

    for i in range(2):
        piped_step(i)
    torch.cuda.synchronize()
    barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    s_in.wait_event(p0)
    for i in range(steps):
        piped_step(i)
    for k in range(2):
        stream.wait_event(ev_out[k])
    p1.record(stream)
    torch.cuda.synchronize()
    p_ms = max_over_ranks(p0.elapsed_time(p1), dev)
    return p_ms, serial_ms, h2d, d2h, h2d_gbs, d2h_gbs


def sustained(run, local, seconds=1.0):
    """Back-to-back steps for about `seconds` with NVML sampling (clocks under load)."""
    import torch
    probe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    probe[0].record(run.stream)
    for _ in range(5):
        run.step()
    probe[1].record(run.stream)
    torch.cuda.synchronize()
    ms = probe[0].elapsed_time(probe[1]) / 5
    n = max(10, int(seconds * 1e3 / max(ms, 1e-3)))
    clocks = ClockSampler()
    clocks.start(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0.record(run.stream)
    for _ in range(n):
        run.step()
    e1.record(run.stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    return {"steps": n, "ms_per_step": e0.elapsed_time(e1) / n, "seconds": t1 - t0,
            "clocks": clocks.stop(t0, t1), "l2": "not flushed (steps back to back)"}


def measure(key, args, rank, world, local, dev, barrier, max_over_ranks):
    """Every measurement of one workload on this rank; rank 0 gets the line dict."""
    import torch
    from koopman_mamba_b200 import _lib
    lib = _lib.lib()
    run = Runner(key, rank, world, dev, lib, _lib)
    wl = run.wl
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    for _ in range(args.warmup):
        run.step()
    torch.cuda.synchronize()
    run.check_status()

    clocks = ClockSampler()
    clocks.start(local)
    dev_ms, t0, t1 = timed_steps(run, args.steps, flush, barrier)
    clock_info = clocks.stop(t0, t1)
    dev_ms_max = max_over_ranks(dev_ms, dev)
    run.check_status()
    job_tokens = wl["B"] * wl["L"] * (world if wl["scaling"] == "weak" else 1)
    value = job_tokens * args.steps / (dev_ms_max / 1e3)
    ms_step = dev_ms_max / args.steps

    kern = per_kernel_ms(run, 5, flush)
    names = run.kernel_names()
    peak, peak_kind = _measured_peak()
    step_algo = run.token_heads * algo_bytes_per_token_head(wl)
    my_ms = dev_ms / args.steps
    achieved = step_algo / (my_ms / 1e3) / 1e9
    traffic = _ncu_traffic(key, names)
    ksum = sum(kern.values())
    roofline = {
        "bound": "hbm", "scope": "step (all kernels of one step, this rank)", "achieved": achieved, "peak": peak,
        "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
        "traffic_ratio": (traffic / step_algo) if traffic else None,
        "algo_bytes": step_algo,
        "algo_model": f"{algo_bytes_per_token_head(wl)} B per token and head ("
                      + ("2*(6r+5P): fwd z,zq,v->y; bwd z,zq,v,dy->dz,dzq,dv" if wl["bwd"]
                         else "2*(2r+2P): z,zq,v->y") + f") x {run.token_heads} token-heads",
        "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
        "dominant_kernel": max(kern, key=kern.get),
        "kernels_ms": {k: round(v, 4) for k, v in kern.items()},
        "kernels_share": {k: round(v / ksum, 4) for k, v in kern.items()},
    }

    e2e = None
    if not args.no_e2e:
        p_ms, serial_ms, h2d, d2h, h2d_gbs, d2h_gbs = e2e_measure(run, args.steps, args.warmup, barrier,
                                                                  max_over_ranks)
        e2e = {"value": job_tokens * args.steps / (p_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h,
               "copies": "double-buffered: host->device and device->host on two copy streams, overlapping "
                         "the neighbouring steps' compute and copies",
               "serial_value": job_tokens * args.steps / (serial_ms / 1e3),
               "rank0_copy_gbs": {"h2d": round(h2d_gbs, 2), "d2h": round(d2h_gbs, 2)}}
    sus = None if args.no_sustained else sustained(run, local)
    run.check_status()
    launches = len(names)
    line = {
        "metric": METRICS[key], "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": wl["scaling"],
        "vs_baseline": None, "dtype": "bf16",
        "compute": "bf16 token tensors; token-level tcgen05 products (fp32 operands as bf16 hi+lo pairs); "
                   "chunk algebra as 3-term-split TF32 mma.sync (fp32-level); fp32 accumulation, Cholesky, "
                   "inverse and power iteration",
        "data": "synthetic (seeded N(0,1)/8 inputs" + (", N(0,1) upstream grad)" if wl["bwd"] else ")"),
        "config": {"workload": wl["name"], "B_per_gpu" if wl["scaling"] == "weak" else "B": wl["B"],
                   "H": wl["H"], "heads_per_rank": run.H, "L": wl["L"], "P": wl["P"], "r": wl["r"],
                   "chunk": wl["CS"], "power_K": wl["K"], "io_dtype": "bf16",
                   "parallelism": (f"dp{world} (batch shards, no collective)" if wl["scaling"] == "weak"
                                   else f"heads split over {world} GPU(s), no collective"),
                   "l2": "flushed between timed steps (256 MiB write outside the events)"},
        "e2e": e2e, "gpu_launches": launches * args.steps, "roofline": roofline, "clocks": clock_info,
        "sustained": sus, "kernel_path": run.path, "wall_s": t1 - t0,
    }
    del run, flush
    torch.cuda.empty_cache()
    return line


def measure_lm(args, rank, world, local, dev, barrier, max_over_ranks):
    """The 50M hybrid Mamba-2 + SKA model's training step (forward, backward with the
    DDP all-reduce over NCCL, AdamW) on synthetic token ids (uniform over the
    vocabulary, seed 3 + 1000 * rank).  The Mamba-2 layers are the package's
    PyTorch stand-in unless mamba_ssm is importable."""
    import torch
    from koopman_mamba_b200.lm import HybridLM, Mamba2Mixer, config_50m_mamba_ska
    B, L = 32, 2048
    cfg = config_50m_mamba_ska()
    torch.manual_seed(3)
    model = HybridLM(cfg).to(dev)
    mamba_kind = "PyTorch Mamba-2 stand-in (mamba_ssm not installed)" \
        if any(isinstance(mm, Mamba2Mixer) for mm in model.modules()) else "mamba_ssm.Mamba2"
    net = model
    if world > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], find_unused_parameters=False)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, fused=True)
    g = torch.Generator().manual_seed(3 + 1000 * rank)
    host_ids = torch.randint(0, cfg.vocab_size, (B, L + 1), generator=g).pin_memory()
    ids = host_ids.to(dev)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def step(x):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = net(x[:, :-1], x[:, 1:])["loss"]
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    clocks = ClockSampler()
    clocks.start(local)
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    losses = []
    for i in range(args.steps):
        ev0[i].record(stream)
        losses.append(step(ids))
        ev1[i].record(stream)
    torch.cuda.synchronize()
    barrier()
    t1 = time.perf_counter()
    clock_info = clocks.stop(t0, t1)
    dev_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(ev0, ev1)), dev)
    tokens = world * B * L
    # end to end: every step copies its token ids in and its loss out
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ea.record(stream)
    for _ in range(args.steps):
        ids.copy_(host_ids, non_blocking=True)
        loss_host.copy_(step(ids).detach(), non_blocking=True)
    eb.record(stream)
    torch.cuda.synchronize()
    e_ms = max_over_ranks(ea.elapsed_time(eb), dev)
    return {
        "metric": "hybrid Mamba-2 + SKA LM training tokens/s (50M model, batch 32 x 2048)", "value": tokens * args.steps / (dev_ms / 1e3),
        "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform token ids, seed 3 + 1000*rank)",
        "config": {"workload": LM_WORKLOAD, "B_per_gpu": B, "L": L, "mamba": mamba_kind,
                   "parallelism": f"DDP over {world} GPU(s), NCCL all-reduce of the gradients"},
        "e2e": {"value": tokens * args.steps / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": host_ids.numel() * 8,
                "d2h_bytes_per_step": 4},
        "loss_first_last": [float(losses[0]), float(losses[-1])],
        "max_memory_gb": torch.cuda.max_memory_allocated(dev) / 1e9, "clocks": clock_info,
        "roofline": None, "cpu_baseline": None, "wall_s": t1 - t0,
    }


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        if args.workload == "lm":
            print(json.dumps({"impl": "reference", "unavailable": "the reference's full model needs mamba_ssm, "
                              "which is not installed on this machine or the GPU box"}), flush=True)
            return 0
        return run_reference_arm(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    want_cpu = (not args.no_cpu_baseline) and world == 1 and rank == 0
    workers = cpu_workers(args.cpu_workers)
    pool = _make_pool(workers) if want_cpu else None   # spawn pool started before any CUDA work

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from koopman_mamba_b200.sharding import max_over_ranks

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    if args.workload == "lm":
        if pool is not None:
            pool.close()
            pool.join()
        line = measure_lm(args, rank, world, local, dev, barrier, max_over_ranks)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(line), flush=True)
        return 0

    keys = [args.workload] + (["c3"] if args.workload == "c2" and not args.no_c3 else [])
    lines = {}
    for key in keys:
        lines[key] = measure(key, args, rank, world, local, dev, barrier, max_over_ranks)
    if want_cpu:
        try:
            for key in keys:
                lines[key]["cpu_baseline"] = cpu_baseline(pool, workers, key)
        finally:
            pool.close()
            pool.join()
    else:
        for key in keys:
            lines[key]["cpu_baseline"] = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line = lines[args.workload]
        if len(keys) > 1:
            sub = lines["c3"]
            line["c3"] = {k: sub[k] for k in ("value", "unit", "ms_per_step", "scaling", "n_gpus", "config",
                                              "roofline", "e2e", "gpu_launches", "cpu_baseline", "clocks",
                                              "sustained", "kernel_path")}
            line["c3"]["metric"] = METRIC_C3
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
