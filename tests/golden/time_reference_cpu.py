"""Time the reference's own CPU path of the SKA core beside the numpy oracle port.

The GPU benchmark's CPU baseline (bench.py ``cpu_baseline`` and ``--impl
reference``) runs the numpy oracle port, because the upstream Python package does
not travel to the GPU machines.  This script calibrates that stand-in: on the
machine where the upstream ``koopman-lm-fast`` checkout is available
(``--ref-root`` or ``SKA_REFERENCE_ROOT``), it times, on the same seeded inputs
and the same cores, the reference's PyTorch CPU path (``backend='pytorch'``:
max-norm scaling, ``_compute_chunk_stats_and_cholesky``, ``_post_cholesky_pytorch``
and its autograd backward, ``koopman_lm/ska.py:73-187,436-457``) and the numpy
port, and prints one JSON line with both throughputs.

Workloads (one series slice each, as the benchmark's CPU legs split them):
  c2  fwd+bwd of one batch element of B=8 H=12 L=2048 P=64 r=32 chunk 64
  c3  fwd of one head of B=1 H=16 L=32768 P=64 r=64 chunk 128

Usage:  python tests/golden/time_reference_cpu.py --ref-root <upstream>/koopman-lm-fast [--threads N]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def _inputs(B, T, H, r, P, seed, dy):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(64)
    out = [torch.randn(B, T, H, n, generator=g) * s for n in (r, r, P)]
    if dy:
        out.append(torch.randn(B, T, H, P, generator=g))
    return [t.bfloat16().float() for t in out]


def _ref_core(ref_ska, z, zq, v, gamma, r, H, P, CS, K):
    max_norm = z.norm(dim=-1, keepdim=True).max(dim=1, keepdim=True)[0].clamp(min=1e-6)
    L, M, C, Q, shapes = ref_ska._compute_chunk_stats_and_cholesky(z / max_norm, zq / max_norm, v, r, H, P, CS, 1e-3)
    return ref_ska._post_cholesky_pytorch(L, M, C, Q, gamma, K, shapes)


def _best(fn, reps):
    fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return min(ts)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref-root", default=os.environ.get("SKA_REFERENCE_ROOT", ""))
    ap.add_argument("--threads", type=int, default=1, help="torch / BLAS threads for both paths")
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    if not a.ref_root or not os.path.isdir(os.path.join(a.ref_root, "koopman_lm")):
        raise SystemExit("pass --ref-root (or set SKA_REFERENCE_ROOT) to the upstream koopman-lm-fast directory")
    sys.path.insert(0, a.ref_root)
    torch.set_num_threads(a.threads)
    from koopman_lm import ska as ref_ska
    from oracle.ska_oracle import SkaParams, ska_core_forward, ska_core_fwd_bwd
    from oracle.ska_torch_port import ska_core_torch

    res = {"threads": a.threads, "reps": a.reps}
    # c2: one batch element, fwd + bwd
    z, zq, v, dy = _inputs(1, 2048, 12, 32, 64, 1, True)

    def ref_c2():
        zz, qq, vv = (t.clone().requires_grad_(True) for t in (z, zq, v))
        gm = torch.tensor(1.0, requires_grad=True)
        _ref_core(ref_ska, zz, qq, vv, gm, 32, 12, 64, 64, 2).backward(dy)

    def torch_c2():
        zz, qq, vv = (t.clone().requires_grad_(True) for t in (z, zq, v))
        gm = torch.tensor(1.0, requires_grad=True)
        ska_core_torch(zz, qq, vv, gm, chunk_size=64).backward(dy)

    npz = [t.numpy() for t in (z, zq, v, dy)]
    port_c2 = lambda: ska_core_fwd_bwd(npz[0], npz[1], npz[2], 1.0, npz[3], SkaParams(), np.float32)  # noqa: E731
    t_ref, t_port, t_torch = _best(ref_c2, a.reps), _best(port_c2, a.reps), _best(torch_c2, a.reps)
    res["c2_one_batch_element_fwd_bwd"] = {"tokens": 2048, "reference_s": t_ref, "numpy_port_s": t_port,
                                           "torch_port_s": t_torch, "reference_tokens_per_s": 2048 / t_ref,
                                           "numpy_port_over_reference": t_ref / t_port,
                                           "torch_port_over_reference": t_ref / t_torch}
    # c3: one head, forward
    z, zq, v = _inputs(1, 32768, 1, 64, 64, 2, False)

    def ref_c3():
        with torch.no_grad():
            _ref_core(ref_ska, z, zq, v, torch.tensor(1.0), 64, 1, 64, 128, 2)

    def torch_c3():
        with torch.no_grad():
            ska_core_torch(z, zq, v, torch.tensor(1.0), chunk_size=128)

    npz = [t.numpy() for t in (z, zq, v)]
    port_c3 = lambda: ska_core_forward(npz[0], npz[1], npz[2], 1.0, SkaParams(chunk_size=128), np.float32)  # noqa: E731
    t_ref, t_port, t_torch = _best(ref_c3, a.reps), _best(port_c3, a.reps), _best(torch_c3, a.reps)
    res["c3_one_head_fwd"] = {"tokens": 32768, "reference_s": t_ref, "numpy_port_s": t_port, "torch_port_s": t_torch,
                              "numpy_port_over_reference": t_ref / t_port,
                              "torch_port_over_reference": t_ref / t_torch}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
