"""Generate golden vectors of the SKA recurrent (decode) path by running the
upstream reference itself.

Runs ``RecurrentKoopmanLM._ska_prefill`` and ``RecurrentKoopmanLM._ska_step``
(``koopman_lm/recurrent.py:129-189`` and ``:270-375``) on one SKA layer of a
seeded ``SKAModule`` (``backend='pytorch'``) wrapped in a pre-norm block whose
norm is the identity, on CPU.  Forward hooks on the projections and on
``out_proj`` record what the reference computed: the prompt's z, zq, v, every
decode token's z_t, zq_t, v_t and the core output y_hat (the input of out_proj,
with eta = 1), next to the state after the prefill and after the last step.
The reference does this math in float32 (``.float()`` upcasts), whatever the
module's dtype.

Writes ``tests/golden/recur_*.npz``.  The upstream ``koopman-lm-fast``
directory is given by ``--ref-root`` or ``SKA_REFERENCE_ROOT``.  The GPU
machines never run this script: they read the committed ``.npz`` files.

Usage:  python tests/golden/make_golden_recurrent.py --ref-root <upstream>/koopman-lm-fast
"""
from __future__ import annotations

import argparse
import os
import sys
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn as nn

REF_ROOT = os.environ.get("SKA_REFERENCE_ROOT", "")
OUT_DIR = os.path.dirname(os.path.abspath(__file__))


class _Block(nn.Module):
    """The reference's SKABlock shape (``model.py:28-49``) with an identity norm,
    so the projections see the raw inputs."""

    def __init__(self, ska):
        super().__init__()
        self.norm = nn.Identity()
        self.ska = ska

    def forward(self, x):
        return x + self.ska(self.norm(x))


def run_case(name, *, B, T, H, r, P, CS, K, gamma, steps, seed, ridge=1e-3):
    sys.path.insert(0, REF_ROOT)
    from koopman_lm import recurrent as ref_rec   # noqa: E402
    from koopman_lm import ska as ref_ska         # noqa: E402

    d_model = H * P
    torch.manual_seed(seed)
    ska = ref_ska.SKAModule(d_model, H, rank=r, head_dim=P, ridge_eps=ridge, power_K=K, chunk_size=CS,
                            backend="pytorch")
    with torch.no_grad():
        ska.eta.fill_(1.0)
        ska.ssn_gamma.fill_(gamma)
    blk = _Block(ska)
    rec = {}

    def grab(key):
        def hook(_m, _inp, out):
            rec.setdefault(key, out.detach().clone())
        return hook

    def grab_in(_m, inp):
        rec.setdefault("y", inp[0].detach().clone())

    hooks = [ska.key_proj.register_forward_hook(grab("z")), ska.query_proj.register_forward_hook(grab("zq")),
             ska.value_proj.register_forward_hook(grab("v")), ska.out_proj.register_forward_pre_hook(grab_in)]
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(B, T, d_model, generator=g) / 4
    self_ = SimpleNamespace(_ska_states={})
    with torch.no_grad():
        _, state = ref_rec.RecurrentKoopmanLM._ska_prefill(self_, blk, x, 0)
    out = dict(z=rec["z"].reshape(B, T, H, r).numpy(), zq=rec["zq"].reshape(B, T, H, r).numpy(),
               v=rec["v"].reshape(B, T, H, P).numpy(),
               G0=state.G.numpy(), M0=state.M.numpy(), C0=state.C_v.numpy(),
               zlast0=state.z_last.numpy(), maxnorm0=state.max_norm.reshape(B, H).numpy())
    self_._ska_states[0] = state
    zs, zqs, vs, ys = [], [], [], []
    for _ in range(steps):
        rec.clear()
        xt = torch.randn(B, 1, d_model, generator=g) / 4
        with torch.no_grad():
            ref_rec.RecurrentKoopmanLM._ska_step(self_, blk, xt, 0)
        zs.append(rec["z"].reshape(B, H, r).numpy())
        zqs.append(rec["zq"].reshape(B, H, r).numpy())
        vs.append(rec["v"].reshape(B, H, P).numpy())
        ys.append(rec["y"].reshape(B, H, P).numpy())
    for h in hooks:
        h.remove()
    st = self_._ska_states[0]
    out.update(z_steps=np.stack(zs), zq_steps=np.stack(zqs), v_steps=np.stack(vs), y_steps=np.stack(ys),
               G1=st.G.numpy(), M1=st.M.numpy(), C1=st.C_v.numpy(), zlast1=st.z_last.numpy())
    meta = dict(B=B, T=T, H=H, r=r, P=P, CS=CS, K=K, gamma=gamma, steps=steps, seed=seed, ridge=ridge)
    for k, val in meta.items():
        out[f"meta_{k}"] = np.asarray(val)
    path = os.path.join(OUT_DIR, f"{name}.npz")
    np.savez_compressed(path, **{k: (v.astype(np.float32) if v.dtype == np.float64 else v) for k, v in out.items()})
    print(f"wrote {path}: y |max| {np.abs(out['y_steps']).max():.3e}")


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "koopman_lm")):
        raise SystemExit("pass --ref-root (or set SKA_REFERENCE_ROOT) to the upstream koopman-lm-fast directory")
    # r = 16 with a ragged last chunk (T % CS != 0), gamma inside the clamp
    run_case("recur_r16", B=2, T=100, H=3, r=16, P=32, CS=32, K=2, gamma=1.2, steps=6, seed=31)
    # r = 32, P = 64 (the benchmark head shape), K = 3, gamma clamped at 1.5
    run_case("recur_r32", B=1, T=200, H=2, r=32, P=64, CS=64, K=3, gamma=1.7, steps=4, seed=32)


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref-root", default=REF_ROOT,
                    help="the upstream koopman-lm-fast directory (default: $SKA_REFERENCE_ROOT)")
    REF_ROOT = ap.parse_args().ref_root
    main()
