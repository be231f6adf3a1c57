"""Generate golden SKA vectors by running the upstream reference itself.

Run where a checkout of the upstream project is available; its
``koopman-lm-fast`` directory is given by ``--ref-root`` or the environment
variable ``SKA_REFERENCE_ROOT``.  Writes ``tests/golden/*.npz``.  The GPU
machines never run this script: they only read the committed ``.npz`` files.

Every case calls the reference's own code with ``backend='pytorch'`` (its
``auto`` backend picks Triton, which cannot run on a CPU), so the gradients
are PyTorch autograd through ``koopman_lm/ska.py:73-187`` (and
``koopman_lm/adaptive_chunking.py:171-256`` for the decay strategy), exactly
what the reference's PyTorch backend trains with.

Core cases replicate ``SKAModule.forward`` between the projections and the
eta/out_proj epilogue (``ska.py:436-457``): fp32 (or fp64) upcast, shared
max-key-norm scaling, chunk statistics + Cholesky, post-Cholesky chain.
The ``module_*`` case runs the whole ``SKAModule`` (projections, eta,
out_proj) with seeded weights and stores its state_dict, so the drop-in
module can be checked end to end.

Usage:  python tests/golden/make_golden.py --ref-root <upstream>/koopman-lm-fast
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np
import torch

REF_ROOT = os.environ.get("SKA_REFERENCE_ROOT", "")
OUT_DIR = os.path.dirname(os.path.abspath(__file__))


def _import_reference():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "koopman_lm")):
        raise SystemExit("pass --ref-root (or set SKA_REFERENCE_ROOT) to the upstream koopman-lm-fast directory")
    sys.path.insert(0, REF_ROOT)
    from koopman_lm import ska as ref_ska                     # noqa: E402
    from koopman_lm import adaptive_chunking as ref_ac        # noqa: E402
    return ref_ska, ref_ac


def ref_core(ref_ska, ref_ac, z, zq, v, gamma, *, r, H, P, CS, ridge, K, decay_alpha):
    """The reference forward between projections and eta (ska.py:436-457)."""
    max_norm = z.norm(dim=-1, keepdim=True).max(dim=1, keepdim=True)[0].clamp(min=1e-6)
    zf = z / max_norm
    zqf = zq / max_norm
    if decay_alpha is None:
        stats = ref_ska._compute_chunk_stats_and_cholesky(zf, zqf, v, r, H, P, CS, ridge)
    else:
        stats = ref_ac.compute_chunk_stats_decay(zf, zqf, v, r, H, P, CS, ridge,
                                                 decay_alpha=decay_alpha)
    L, M, C, Q, shapes = stats
    y = ref_ska._post_cholesky_pytorch(L, M, C, Q, gamma, K, shapes)
    return y


def make_inputs(B, T, H, r, P, seed, *, scale_dim, bf16_round=False, dtype=torch.float32):
    """z, zq, v ~ N(0,1)/sqrt(scale_dim) then dy ~ N(0,1), one generator, in
    that order (z, zq, v, dy)."""
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(scale_dim)
    z = torch.randn(B, T, H, r, generator=g) * s
    zq = torch.randn(B, T, H, r, generator=g) * s
    v = torch.randn(B, T, H, P, generator=g) * s
    dy = torch.randn(B, T, H, P, generator=g)
    if bf16_round:
        z, zq, v, dy = (t.to(torch.bfloat16).float() for t in (z, zq, v, dy))
    return [t.to(dtype) for t in (z, zq, v, dy)]


def run_core_case(ref_ska, ref_ac, name, *, B, T, H, r, P, CS, ridge=1e-3, K=2,
                  gamma=1.0, decay_alpha=None, seed=0, scale_dim=64, bf16_round=False,
                  mutate=None, also_fp32=False, note=""):
    out = {}
    truth = None
    for dt, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
        if tag == "f32" and not also_fp32:
            continue
        z, zq, v, dy = make_inputs(B, T, H, r, P, seed, scale_dim=scale_dim,
                                   bf16_round=bf16_round, dtype=torch.float32)
        if mutate is not None:
            z, zq, v = mutate(z, zq, v)
        if tag == "f64":
            out.update(z=z.numpy(), zq=zq.numpy(), v=v.numpy(), dy=dy.numpy())
        z, zq, v, dy = (t.to(dt) for t in (z, zq, v, dy))
        z.requires_grad_(True)
        zq.requires_grad_(True)
        v.requires_grad_(True)
        gm = torch.tensor(gamma, dtype=dt, requires_grad=True)
        y = ref_core(ref_ska, ref_ac, z, zq, v, gm, r=r, H=H, P=P, CS=CS, ridge=ridge, K=K,
                     decay_alpha=decay_alpha)
        y.backward(dy)
        res = dict(y=y.detach().numpy(), dz=z.grad.numpy(), dzq=zq.grad.numpy(),
                   dv=v.grad.numpy(), dgamma=np.asarray(gm.grad.item()))
        if tag == "f64":
            # stored as float32: the pin tolerance (~1e-6) is far above its rounding
            for k, val in res.items():
                out[f"{k}_f64"] = val.astype(np.float32) if val.ndim else val
            truth = res
        else:
            # the reference's own fp32 error against its fp64 run, as scalars
            for k in ("y", "dz", "dzq", "dv"):
                a, b = res[k].astype(np.float64), truth[k]
                out[f"ref_f32_relerr_{k}"] = np.asarray(
                    np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
    meta = dict(B=B, T=T, H=H, r=r, P=P, CS=CS, ridge=ridge, K=K, gamma=gamma,
                decay_alpha=(-1.0 if decay_alpha is None else decay_alpha), seed=seed,
                bf16_round=int(bf16_round))
    for k, val in meta.items():
        out[f"meta_{k}"] = np.asarray(val)
    out["meta_note"] = np.asarray(note)
    path = os.path.join(OUT_DIR, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: y_f64 |max| {np.abs(out['y_f64']).max():.3e}  dgamma {out['dgamma_f64']}")


def run_module_case(ref_ska, name, *, B, T, d_model, H, r, CS, seed, dtype=torch.float64, bf16_proj=False):
    """Whole SKAModule (backend='pytorch') with seeded non-zero weights.

    bf16_proj: the key/query/value projection outputs are rounded to bfloat16 (a
    straight-through rounding: the backward passes the gradient unchanged), which is
    what those projections produce under torch.autocast(bfloat16) on a GPU while
    the reference's core itself runs with autocast disabled (ska.py:433-457)."""
    torch.manual_seed(seed)
    m = ref_ska.SKAModule(d_model, H, rank=r, chunk_size=CS, backend="pytorch").to(dtype)
    if bf16_proj:
        def _round(_mod, _inp, out):
            return out + (out.to(torch.bfloat16).to(out.dtype) - out).detach()
        for proj in (m.key_proj, m.query_proj, m.value_proj):
            proj.register_forward_hook(_round)
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        m.out_proj.weight.copy_(torch.randn(m.out_proj.weight.shape, generator=g).to(dtype)
                                / math.sqrt(m.out_proj.weight.shape[1]))
        m.ssn_gamma.fill_(1.1)
    x = (torch.randn(B, T, d_model, generator=g)).to(dtype).requires_grad_(True)
    dout = torch.randn(B, T, d_model, generator=g).to(dtype)
    out = m(x)
    out.backward(dout)
    f32 = lambda t: t.detach().to(torch.float32).numpy()   # noqa: E731
    res = {f"sd_{k}": f32(v) for k, v in m.state_dict().items()}
    res.update(x=f32(x), dout=f32(dout), out=f32(out), dx=f32(x.grad))
    for pname, p in m.named_parameters():
        res[f"grad_{pname}"] = f32(p.grad)
    meta = dict(B=B, T=T, d_model=d_model, H=H, r=r, CS=CS, seed=seed)
    for k, val in meta.items():
        res[f"meta_{k}"] = np.asarray(val)
    path = os.path.join(OUT_DIR, f"{name}.npz")
    np.savez_compressed(path, **res)
    print(f"wrote {path}: out |max| {np.abs(res['out']).max():.3e}")


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref_ska, ref_ac = _import_reference()

    # Config 1 (the reference's CPU-runnable case): B=2 H=4 L=512 d=64 r=16,
    # ridge 1e-3, chunk 64, seed 0; fp32 and fp64 reference runs.
    run_core_case(ref_ska, ref_ac, "core_cfg1", B=2, T=512, H=4, r=16, P=64, CS=64, seed=0,
                  also_fp32=True, note="config 1: fp32 reference path")
    # Ragged T (T % CS != 0), gamma strictly inside the clamp.
    run_core_case(ref_ska, ref_ac, "core_pad", B=1, T=200, H=3, r=16, P=32, CS=64, seed=11,
                  gamma=1.2, note="T % CS != 0 (zero padded tail)")
    # Library default rank 48 (not a power of two), gamma at the upper clamp bound.
    run_core_case(ref_ska, ref_ac, "core_r48", B=1, T=256, H=2, r=48, P=64, CS=64, seed=12,
                  gamma=1.5, note="r=48, gamma=1.5 (inclusive upper clamp)")
    # Decay strategy (adaptive_chunking.compute_chunk_stats_decay).
    run_core_case(ref_ska, ref_ac, "core_decay", B=1, T=320, H=2, r=16, P=32, CS=64, seed=13,
                  gamma=1.3, decay_alpha=0.9, note="chunk_strategy='decay', alpha=0.9")

    # Jitter path: negative ridge makes chunk 0 (G = ridge*I) fail, and zeroed
    # key dimensions make later slices fail too; jitter 1e-4 repairs both.
    def zero_dims(z, zq, v):
        z = z.clone()
        z[..., -3:] = 0.0
        return z, zq, v
    run_core_case(ref_ska, ref_ac, "core_jitter", B=1, T=256, H=2, r=16, P=32, CS=64, seed=14,
                  ridge=-5e-5, gamma=1.7, mutate=zero_dims,
                  note="negative ridge + rank-deficient keys: jitter branch; gamma clamped (dgamma=0)")
    # A single chunk (T < CS): chunk 0 outputs are exactly zero.
    run_core_case(ref_ska, ref_ac, "core_onechunk", B=2, T=40, H=2, r=16, P=32, CS=64, seed=15,
                  note="T < CS: one chunk, y == 0")
    # Other filter powers and chunk sizes.
    run_core_case(ref_ska, ref_ac, "core_k3", B=1, T=256, H=2, r=16, P=16, CS=32, seed=16, K=3,
                  gamma=1.25, note="power_K=3, CS=32")
    run_core_case(ref_ska, ref_ac, "core_k1", B=1, T=192, H=2, r=32, P=32, CS=64, seed=17, K=1,
                  gamma=1.1, note="power_K=1")
    # Config-2-like numerics: bf16-rounded inputs, r=32, P=64.
    run_core_case(ref_ska, ref_ac, "core_bf16in", B=1, T=256, H=2, r=32, P=64, CS=64, seed=1,
                  bf16_round=True, note="bf16-rounded inputs, r=32 P=64 (config 2 class)")
    # Config-3 class: r=64, CS=128.
    run_core_case(ref_ska, ref_ac, "core_r64", B=1, T=512, H=1, r=64, P=64, CS=128, seed=2,
                  bf16_round=True, note="r=64 CS=128 (config 3 class)")
    # Whole module: projections + core + eta + out_proj.
    run_module_case(ref_ska, "module_small", B=2, T=200, d_model=128, H=2, r=16, CS=64, seed=21)
    # The same module with bf16-rounded projections (the autocast(bfloat16) setting).
    run_module_case(ref_ska, "module_small_bf16proj", B=2, T=200, d_model=128, H=2, r=16, CS=64, seed=21,
                    bf16_proj=True)


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref-root", default=REF_ROOT,
                    help="the upstream koopman-lm-fast directory (default: $SKA_REFERENCE_ROOT)")
    REF_ROOT = ap.parse_args().ref_root
    main()
