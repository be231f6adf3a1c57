"""PyTorch CPU restatement of the SKA core: the timed CPU baseline.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module: only
``tests/`` (which check it against the numpy oracle) and the CPU legs of
``bench.py`` (``cpu_baseline`` and ``--impl reference``) use it.

Why it exists: the upstream package cannot travel to the GPU machines, and its
CPU path is PyTorch on the host cores (``backend='pytorch'``: batched LAPACK
Cholesky, triangular solves, einsums, ``cumsum``, autograd for the backward).
The numpy oracle restates the same algorithm with written-out loops and is 2-4x
slower than that path on the same core (``tests/golden/time_reference_cpu.py``
measures both), so timing it would flatter the GPU.  This module is the oracle's
op sequence (``oracle/ska_oracle.py:ska_core_forward``, which cites
``KLF/koopman_lm/ska.py:41-187`` line by line) on torch tensors, fp32 on the CPU,
with autograd for the backward, as the reference's own CPU path computes it.
"""
from __future__ import annotations

import math

import torch

__all__ = ["ska_core_torch"]


def _power_normalize(A, n_iters=6):
    """``ska.py:41-58``: power iteration from v = 1/sqrt(r) under no_grad, then
    A / max(sigma, 1) with the scale a constant for the backward."""
    with torch.no_grad():
        v = torch.ones(*A.shape[:-1], 1, dtype=A.dtype) / math.sqrt(A.shape[-1])
        for _ in range(n_iters):
            u = A @ v
            u = u / u.norm(dim=-2, keepdim=True).clamp(min=1e-8)
            v = A.transpose(-1, -2) @ u
            v = v / v.norm(dim=-2, keepdim=True).clamp(min=1e-8)
        sigma = (A @ v).norm(dim=-2).squeeze(-1)
        scale = sigma.clamp(min=1.0)
    return A / scale[..., None, None]


def ska_core_torch(z, zq, v, gamma, *, chunk_size=64, ridge_eps=1e-3, power_K=2, jitter=1e-4):
    """``(z, zq, v, gamma) -> y`` for [B,T,H,r] / [B,T,H,P] float tensors on the CPU
    (differentiable through autograd)."""
    B, T, H, r = z.shape
    P = v.shape[-1]
    CS = chunk_size
    nrm = z.norm(dim=-1, keepdim=True)                              # [B,T,H,1]
    m = nrm.max(dim=1, keepdim=True)[0].clamp(min=1e-6)            # ska.py:441
    zn, zqn = z / m, zq / m
    C = (T + CS - 1) // CS
    pad = C * CS - T
    if pad:
        zn, zqn, v = (torch.nn.functional.pad(t, (0, 0, 0, 0, 0, pad)) for t in (zn, zqn, v))
    zc = zn.reshape(B, C, CS, H, r)
    zqc = zqn.reshape(B, C, CS, H, r)
    vc = v.reshape(B, C, CS, H, P)
    G = torch.einsum("bcthr,bcths->bchrs", zc, zc)                # ska.py:102-111
    M = torch.einsum("bcthr,bcths->bchrs", zc[:, :, 1:], zc[:, :, :-1])
    Cs = torch.einsum("bcthp,bcthr->bchpr", vc, zc)

    def excl(x):                                                    # ska.py:114-133
        return torch.cat([torch.zeros_like(x[:, :1]), torch.cumsum(x, dim=1)[:, :-1]], dim=1)

    Gx = excl(G) + ridge_eps * torch.eye(r, dtype=z.dtype)
    Mx = excl(M)
    if C > 1:   # boundary transition into chunk c >= 1, counted from chunk c on (inclusive)
        bnd = torch.einsum("bchr,bchs->bchrs", zc[:, 1:, 0], zc[:, :-1, -1])
        Mx = Mx + torch.cat([torch.zeros_like(bnd[:, :1]), torch.cumsum(bnd, dim=1)], dim=1)
    Cx = excl(Cs)
    N = B * C * H
    Gf = Gx.reshape(N, r, r)
    Gs = 0.5 * (Gf + Gf.transpose(-1, -2))
    L, info = torch.linalg.cholesky_ex(Gs)
    bad = info > 0
    if bool(bad.any()):
        Lj, _ = torch.linalg.cholesky_ex(Gs + jitter * torch.eye(r, dtype=z.dtype))
        L = torch.where(bad[:, None, None], Lj, L)
    Mf = Mx.reshape(N, r, r)
    Cf = Cx.reshape(N, P, r)
    Qf = zqc.permute(0, 1, 3, 4, 2).reshape(N, r, CS)
    A = torch.cholesky_solve(Mf.transpose(-1, -2), L).transpose(-1, -2)
    A = _power_normalize(A) * gamma.clamp(1.0, 1.5)
    Bv = torch.cholesky_solve(Cf.transpose(-1, -2), L).transpose(-1, -2)
    w = torch.linalg.solve_triangular(L, Qf, upper=False)
    for _ in range(power_K):
        w = A @ w
    y = Bv @ (L @ w)
    return y.reshape(B, C, H, P, CS).permute(0, 1, 4, 2, 3).reshape(B, C * CS, H, P)[:, :T]
