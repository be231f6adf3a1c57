"""CPU oracle for the Spectral Koopman Attention (SKA) core: numpy restatement.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use it, and only as the checker (or as the timed CPU stand-in
for the reference's own CPU path).  The CUDA library never routes through it.

What it restates (paths relative to the upstream project root, ``KLF`` =
``koopman-lm-fast``):

* forward, ``chunk_strategy='standard'``:
  ``KLF/koopman_lm/ska.py:436-443`` (fp32 upcast + shared max key norm),
  ``ska.py:87-99`` (zero pad + chunk reshape), ``ska.py:102-111`` (per-chunk
  Gram / transition / value statistics and boundary transitions),
  ``ska.py:114-133`` (exclusive prefix sums + ridge), ``ska.py:136-145``
  (symmetrise, Cholesky, jitter on failing slices), ``ska.py:165-187``
  (post-Cholesky solves, spectral normalisation ``ska.py:41-58``, gamma clamp,
  filter ``ska.py:61-66``, readout, un-chunk);
* forward, ``chunk_strategy='decay'``: the alpha-weighted exclusive scan of
  ``KLF/koopman_lm/adaptive_chunking.py:213-238``;
* backward: the reference has no hand-written backward; its gradients are
  PyTorch autograd through the ops above.  ``ska_core_backward`` is the
  reverse-mode chain rule through the same op sequence, one vector-Jacobian
  product per reference op, in reverse order, using the VJP conventions of
  the PyTorch ops the reference calls (``cholesky_ex``, ``cholesky_solve``,
  ``solve_triangular``, ``clamp`` (inclusive bounds), ``max(dim)`` (gradient
  to the arg-max token), ``norm``).

Linear algebra is written out (column Cholesky with per-slice failure info,
forward/back substitution) so that the oracle needs numpy only and reports
the same per-slice ``info`` that ``torch.linalg.cholesky_ex`` reports.

Parity pin: ``tests/golden/make_golden.py`` runs the upstream module itself
(``backend='pytorch'``) on seeded inputs and stores inputs, outputs and
autograd gradients under ``tests/golden/``; ``tests/test_oracle.py`` checks
this oracle against every stored case.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

__all__ = [
    "SkaParams",
    "cholesky_ex",
    "ska_core_forward",
    "ska_core_backward",
    "ska_core_fwd_bwd",
    "rel_fro",
]


@dataclass(frozen=True)
class SkaParams:
    """Static SKA-core parameters (constructor arguments of the reference
    ``SKAModule``, ``KLF/koopman_lm/ska.py:368-371``)."""

    chunk_size: int = 64
    ridge_eps: float = 1e-3
    power_K: int = 2
    # None = 'standard' strategy; a float = 'decay' strategy with that alpha.
    decay_alpha: float | None = None
    # Number of power iterations in the spectral normalisation (ska.py:41).
    power_iters: int = 6
    # Jitter added to failing Cholesky slices (ska.py:142).
    jitter: float = 1e-4


def rel_fro(a, b) -> float:
    """Norm-relative error ||a-b||_F / ||b||_F (0 when both are zero)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    if den == 0.0:
        return float(num)
    return float(num / den)


# ----------------------------------------------------------------------------
# Small batched linear algebra (restating the LAPACK/PyTorch ops used upstream)
# ----------------------------------------------------------------------------

def cholesky_ex(G: np.ndarray):
    """Batched lower Cholesky with per-slice failure report.

    Same contract as ``torch.linalg.cholesky_ex`` as called at
    ``KLF/koopman_lm/ska.py:140``: reads the lower triangle, returns ``(L,
    info)`` with ``info[n] = j+1`` for the first non-positive pivot ``j`` of
    slice ``n`` (0 when the factorisation succeeded).  Column-oriented
    (left-looking) factorisation, as in LAPACK's unblocked ``potf2``.
    """
    G = np.asarray(G)
    N, r, _ = G.shape
    L = np.zeros_like(G)
    info = np.zeros(N, dtype=np.int64)
    for j in range(r):
        # s[:, i] = G[i, j] - sum_{k<j} L[i, k] L[j, k]   for i >= j
        s = G[:, j:, j] - np.einsum("nik,nk->ni", L[:, j:, :j], L[:, j, :j])
        d = s[:, 0]
        ok = d > 0
        newly_bad = (~ok) & (info == 0)
        info[newly_bad] = j + 1
        with np.errstate(invalid="ignore", divide="ignore"):
            ljj = np.sqrt(np.where(ok, d, np.nan))
            L[:, j, j] = ljj
            if j + 1 < r:
                L[:, j + 1:, j] = s[:, 1:] / ljj[:, None]
    return L, info


def _solve_lower(L: np.ndarray, B: np.ndarray) -> np.ndarray:
    """X = L^{-1} B for lower-triangular L (forward substitution)."""
    N, r, _ = L.shape
    X = np.zeros(np.broadcast_shapes(B.shape), dtype=np.result_type(L, B))
    for i in range(r):
        acc = B[:, i, :] - np.einsum("nk,nkc->nc", L[:, i, :i], X[:, :i, :])
        X[:, i, :] = acc / L[:, i, i][:, None]
    return X


def _solve_upper_t(L: np.ndarray, B: np.ndarray) -> np.ndarray:
    """X = L^{-T} B for lower-triangular L (back substitution on L^T)."""
    N, r, _ = L.shape
    X = np.zeros(np.broadcast_shapes(B.shape), dtype=np.result_type(L, B))
    for i in range(r - 1, -1, -1):
        acc = B[:, i, :] - np.einsum("nk,nkc->nc", L[:, i + 1:, i], X[:, i + 1:, :])
        X[:, i, :] = acc / L[:, i, i][:, None]
    return X


def _cholesky_solve(B: np.ndarray, L: np.ndarray) -> np.ndarray:
    """X = (L L^T)^{-1} B, i.e. ``torch.cholesky_solve(B, L)``."""
    return _solve_upper_t(L, _solve_lower(L, B))


def _mT(x: np.ndarray) -> np.ndarray:
    return np.swapaxes(x, -1, -2)


def _spectral_normalize(A: np.ndarray, n_iters: int):
    """``_spectral_normalize_power_iter`` (``ska.py:41-58``): power iteration
    from v = 1/sqrt(r), returns ``(A / max(sigma, 1), sigma, scale)``.  The
    scale is a constant for the backward (the loop runs under no_grad)."""
    N, r, _ = A.shape
    v = np.ones((N, r, 1), dtype=A.dtype) / np.asarray(math.sqrt(r), dtype=A.dtype)
    tiny = np.asarray(1e-8, dtype=A.dtype)
    for _ in range(n_iters):
        Av = A @ v
        u = Av / np.maximum(np.linalg.norm(Av, axis=-2, keepdims=True), tiny)
        Atu = _mT(A) @ u
        v = Atu / np.maximum(np.linalg.norm(Atu, axis=-2, keepdims=True), tiny)
    sigma = np.linalg.norm(A @ v, axis=-2)[..., 0]
    scale = np.maximum(sigma, np.asarray(1.0, dtype=A.dtype))
    return A / scale[:, None, None], sigma, scale


# ----------------------------------------------------------------------------
# Forward
# ----------------------------------------------------------------------------

def _exclusive_scan(X: np.ndarray, alpha: float | None) -> np.ndarray:
    """Exclusive prefix over the chunk axis (axis 1).

    ``alpha is None``: ``cumsum`` then shift (``ska.py:116-118``).
    ``alpha`` given: ``excl[c] = alpha * excl[c-1] + X[c-1]``
    (``adaptive_chunking.py:225-234``).
    """
    out = np.zeros_like(X)
    if alpha is None:
        if X.shape[1] > 1:
            out[:, 1:] = np.cumsum(X, axis=1)[:, :-1]
        return out
    acc = np.zeros_like(X[:, 0])
    a = np.asarray(alpha, dtype=X.dtype)
    for c in range(X.shape[1]):
        out[:, c] = acc
        acc = a * acc + X[:, c]
    return out


def ska_core_forward(z, zq, v, gamma, params: SkaParams = SkaParams(),
                     dtype=np.float64):
    """SKA core forward: ``(z, zq, v, gamma) -> y_hat`` of shape [B,T,H,P].

    ``z, zq``: [B,T,H,r]; ``v``: [B,T,H,P]; ``gamma``: the ``ssn_gamma``
    scalar.  Everything is computed in ``dtype`` (the reference computes in
    fp32 after ``.float()`` at ``ska.py:436-438``; float64 gives the
    tie-breaking "truth").  Returns ``(y, cache)``; ``cache`` feeds
    :func:`ska_core_backward`.
    """
    z = np.asarray(z, dtype=dtype)
    zq = np.asarray(zq, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    B, T, H, r = z.shape
    P = v.shape[-1]
    CS = params.chunk_size
    if T <= 0:
        raise ValueError("SKA core needs T >= 1 (the reference's max over T fails on T=0)")

    # ska.py:441-443: m = max_t ||z_t||, clamped, shared by keys and queries.
    nrm = np.sqrt(np.sum(z * z, axis=-1))                       # [B,T,H]
    t_star = np.argmax(nrm, axis=1)                             # [B,H] first max
    raw_max = np.take_along_axis(nrm, t_star[:, None, :], axis=1)[:, 0, :]
    m = np.maximum(raw_max, np.asarray(1e-6, dtype=dtype))      # [B,H]
    zn = z / m[:, None, :, None]
    zqn = zq / m[:, None, :, None]

    # ska.py:87-99: zero pad to C*CS, chunk reshape.
    C = (T + CS - 1) // CS
    Tp = C * CS
    pad = Tp - T

    def _pad(x):
        if pad == 0:
            return x
        return np.concatenate([x, np.zeros((B, pad) + x.shape[2:], dtype=x.dtype)], axis=1)

    zc = _pad(zn).reshape(B, C, CS, H, r)
    zqc = _pad(zqn).reshape(B, C, CS, H, r)
    vc = _pad(v).reshape(B, C, CS, H, P)

    # ska.py:102-111: per-chunk statistics + boundary transitions.
    Gch = np.einsum("bcthr,bcths->bchrs", zc, zc, optimize=True)
    Mch = np.einsum("bcthr,bcths->bchrs", zc[:, :, 1:], zc[:, :, :-1], optimize=True)
    Cch = np.einsum("bcthp,bcthr->bchpr", vc, zc, optimize=True)
    Mbnd = np.zeros((B, C, H, r, r), dtype=dtype)
    if C > 1:
        # Mbnd[c] = z_first(c) z_last(c-1)^T for c >= 1
        Mbnd[:, 1:] = np.einsum("bchr,bchs->bchrs", zc[:, 1:, 0], zc[:, :-1, -1], optimize=True)

    # ska.py:114-133 (standard) / adaptive_chunking.py:225-238 (decay).
    alpha = params.decay_alpha
    eye = np.eye(r, dtype=dtype)
    Gx = _exclusive_scan(Gch, alpha) + np.asarray(params.ridge_eps, dtype=dtype) * eye
    if alpha is None:
        # M_excl[c] = sum_{c'<c} M[c'] + sum_{c'<=c} Mbnd[c']
        Mx = _exclusive_scan(Mch, None) + np.cumsum(Mbnd, axis=1)
    else:
        # decay: the boundary into chunk c'+1 is added right after chunk c'
        # (adaptive_chunking.py:236-238), so it decays with chunk c''s stats.
        Mshift = Mch.copy()
        if C > 1:
            Mshift[:, :-1] += Mbnd[:, 1:]
        Mx = _exclusive_scan(Mshift, alpha)
    Cx = _exclusive_scan(Cch, alpha)

    # ska.py:136-145: symmetrise, Cholesky, jitter on failing slices.
    N = B * C * H
    Gf = Gx.reshape(N, r, r)
    Gs = np.asarray(0.5, dtype=dtype) * (Gf + _mT(Gf))
    L0, info = cholesky_ex(Gs)
    Lj, _ = cholesky_ex(Gs + np.asarray(params.jitter, dtype=dtype) * eye)
    fix = info > 0
    L = np.where(fix[:, None, None], Lj, L0)

    Mf = Mx.reshape(N, r, r)
    Cf = Cx.reshape(N, P, r)
    Qf = np.ascontiguousarray(np.transpose(zqc, (0, 1, 3, 4, 2))).reshape(N, r, CS)

    # ska.py:165-169: A_w = M G^{-1}, spectral norm, gamma clamp.
    AwT = _cholesky_solve(_mT(Mf), L)
    Aw0 = _mT(AwT)
    Awn, sigma, sscale = _spectral_normalize(Aw0, params.power_iters)
    g = float(np.asarray(gamma, dtype=np.float64))
    gsafe = np.asarray(min(max(g, 1.0), 1.5), dtype=dtype)
    A = Awn * gsafe

    # ska.py:172-176
    BvT = _cholesky_solve(_mT(Cf), L)
    Bv = _mT(BvT)
    wq = _solve_lower(L, Qf)

    # ska.py:179-181 (filter ska.py:61-66)
    res = [wq]
    for _ in range(params.power_K):
        res.append(A @ res[-1])
    wf = res[-1]
    zo = L @ wf
    yf = Bv @ zo

    # ska.py:183-186
    y = np.transpose(yf.reshape(B, C, H, P, CS), (0, 1, 4, 2, 3)).reshape(B, Tp, H, P)[:, :T]

    cache = dict(
        shape=(B, T, H, r, P, C, CS, pad), params=params, dtype=dtype,
        z=z, zq=zq, v=v, nrm=nrm, t_star=t_star, raw_max=raw_max, m=m,
        zc=zc, zqc=zqc, vc=vc, L=L, info=info, Mf=Mf, Cf=Cf, Qf=Qf,
        AwT=AwT, Awn=Awn, sigma=sigma, sscale=sscale, g=g, gsafe=gsafe, A=A,
        BvT=BvT, Bv=Bv, res=res, wf=wf, zo=zo,
    )
    return np.ascontiguousarray(y), cache


# ----------------------------------------------------------------------------
# Backward (reverse mode through the same op sequence)
# ----------------------------------------------------------------------------

def _chol_solve_vjp(gX, X, L):
    """VJP of ``X = cholesky_solve(Bm, L)``: returns (gB, gL) with PyTorch's
    convention gB = (LL^T)^{-1} gX, gL = -(gB X^T + X gB^T) L."""
    gB = _cholesky_solve(gX, L)
    common = gB @ _mT(X)
    common = common + _mT(common)
    return gB, -(common @ L)


def _cholesky_vjp(gL, L):
    """VJP of ``L = cholesky(A)`` (Murray 2016, as PyTorch implements it):
    P = tril(L^T gL); P = (P + tril(P,-1)^T)/2; gA = L^{-T} P L^{-1}."""
    Pm = np.tril(_mT(L) @ gL)
    Pm = 0.5 * (Pm + _mT(np.tril(Pm, -1)))
    # gA = L^{-T} Pm L^{-1}  =  solve_upper_t(L, (solve_upper_t(L, Pm^T))^T)
    X = _solve_upper_t(L, Pm)          # L^{-T} Pm
    gA = _mT(_solve_upper_t(L, _mT(X)))  # (L^{-T} (L^{-T} Pm)^T)^T = L^{-T} Pm L^{-1}
    return gA


def _exclusive_scan_vjp(gX: np.ndarray, alpha: float | None) -> np.ndarray:
    """Adjoint of :func:`_exclusive_scan` (reverse exclusive suffix sum)."""
    out = np.zeros_like(gX)
    Cn = gX.shape[1]
    if alpha is None:
        if Cn > 1:
            rev = np.cumsum(gX[:, ::-1], axis=1)[:, ::-1]   # inclusive suffix
            out[:, :-1] = rev[:, 1:]
        return out
    a = np.asarray(alpha, dtype=gX.dtype)
    acc = np.zeros_like(gX[:, 0])
    for c in range(Cn - 1, -1, -1):
        out[:, c] = acc
        acc = a * acc + gX[:, c]
    return out


def ska_core_backward(dy, cache):
    """Gradients ``(dz, dzq, dv, dgamma)`` of ``<dy, y>`` w.r.t. the core's
    inputs, following PyTorch autograd through ``ska.py:436-187``."""
    B, T, H, r, P, C, CS, pad = cache["shape"]
    params: SkaParams = cache["params"]
    dtype = cache["dtype"]
    N = B * C * H
    L = cache["L"]
    dy = np.asarray(dy, dtype=dtype)

    # un-chunk (ska.py:183-186)
    dyp = np.zeros((B, C * CS, H, P), dtype=dtype)
    dyp[:, :T] = dy
    dyf = np.ascontiguousarray(np.transpose(dyp.reshape(B, C, CS, H, P), (0, 1, 3, 4, 2))).reshape(N, P, CS)

    # y_flat = B_v @ z_out ; z_out = L @ w_f  (ska.py:180-181)
    Bv, zo, wf = cache["Bv"], cache["zo"], cache["wf"]
    gBv = dyf @ _mT(zo)
    gzo = _mT(Bv) @ dyf
    gL = gzo @ _mT(wf)
    gres = _mT(L) @ gzo

    # filter (ska.py:61-66): res_{k+1} = A res_k
    A, res = cache["A"], cache["res"]
    gA = np.zeros_like(A)
    for k in range(params.power_K - 1, -1, -1):
        gA += gres @ _mT(res[k])
        gres = _mT(A) @ gres
    gwq = gres

    # w_q = solve_triangular(L, zq_flat) (ska.py:176)
    wq = res[0]
    gQ = _solve_upper_t(L, gwq)
    gL += np.tril(-(gQ @ _mT(wq)))

    # B_v = cholesky_solve(C^T, L)^T (ska.py:172-173)
    gBvT = _mT(gBv)
    gCT, gL_b = _chol_solve_vjp(gBvT, cache["BvT"], L)
    gL += gL_b
    gCf = _mT(gCT)

    # A = Awn * clamp(gamma) ; Awn = Aw0 / scale (scale constant) (ska.py:167-169)
    Awn, gsafe, g = cache["Awn"], cache["gsafe"], cache["g"]
    dgsafe = float(np.sum(gA * Awn, dtype=np.float64))
    dgamma = dgsafe if (1.0 <= g <= 1.5) else 0.0
    gAw0 = gA * gsafe / cache["sscale"][:, None, None]

    # A_w = cholesky_solve(M^T, L)^T (ska.py:165-166)
    gAwT = _mT(gAw0)
    gMT, gL_a = _chol_solve_vjp(gAwT, cache["AwT"], L)
    gL += gL_a
    gMf = _mT(gMT)

    # L = cholesky(G_sym) (jittered slices: same VJP evaluated at their L)
    gGs = _cholesky_vjp(gL, L)
    # G_sym = (G + G^T)/2
    gGx = 0.5 * (gGs + _mT(gGs))

    gGx = gGx.reshape(B, C, H, r, r)
    gMx = gMf.reshape(B, C, H, r, r)
    gCx = gCf.reshape(B, C, H, P, r)

    # prefix scans (ska.py:114-133 / adaptive_chunking.py:225-238)
    alpha = params.decay_alpha
    gGch = _exclusive_scan_vjp(gGx, alpha)
    gCch = _exclusive_scan_vjp(gCx, alpha)
    if alpha is None:
        gMch = _exclusive_scan_vjp(gMx, None)
        gMbnd = np.cumsum(gMx[:, ::-1], axis=1)[:, ::-1]    # adjoint of inclusive cumsum
    else:
        gMshift = _exclusive_scan_vjp(gMx, alpha)
        gMch = gMshift
        gMbnd = np.zeros_like(gMx)
        if C > 1:
            gMbnd[:, 1:] = gMshift[:, :-1]

    # einsums (ska.py:102-111)
    zc, vc = cache["zc"], cache["vc"]
    gzc = np.einsum("bchrs,bcths->bcthr", gGch + np.swapaxes(gGch, -1, -2), zc, optimize=True)
    gzc[:, :, 1:] += np.einsum("bchrs,bcths->bcthr", gMch, zc[:, :, :-1], optimize=True)
    gzc[:, :, :-1] += np.einsum("bchrs,bcthr->bcths", gMch, zc[:, :, 1:], optimize=True)
    gzc += np.einsum("bchpr,bcthp->bcthr", gCch, vc, optimize=True)
    gvc = np.einsum("bchpr,bcthr->bcthp", gCch, zc, optimize=True)
    if C > 1:
        gzc[:, 1:, 0] += np.einsum("bchrs,bchs->bchr", gMbnd[:, 1:], zc[:, :-1, -1], optimize=True)
        gzc[:, :-1, -1] += np.einsum("bchrs,bchr->bchs", gMbnd[:, 1:], zc[:, 1:, 0], optimize=True)

    # zq_flat = permute(zq_c) ; un-pad
    gzqc = np.transpose(gQ.reshape(B, C, H, r, CS), (0, 1, 4, 2, 3))
    gzn = gzc.reshape(B, C * CS, H, r)[:, :T]
    gzqn = np.ascontiguousarray(gzqc).reshape(B, C * CS, H, r)[:, :T]
    gv = np.ascontiguousarray(gvc.reshape(B, C * CS, H, P)[:, :T])

    # z_f / max_norm, zq_f / max_norm (ska.py:442-443)
    z, zq, m = cache["z"], cache["zq"], cache["m"]
    mb = m[:, None, :, None]
    gz = gzn / mb
    gzq = gzqn / mb
    gm = -(np.sum(gzn * z, axis=(1, 3)) + np.sum(gzqn * zq, axis=(1, 3))) / (m * m)   # [B,H]

    # max_norm = norm(z).max(dim=1).clamp(min=1e-6): gradient reaches the
    # arg-max token when the clamp is inactive (x >= min passes, inclusive).
    raw_max, t_star, nrm = cache["raw_max"], cache["t_star"], cache["nrm"]
    pass_mask = raw_max >= 1e-6
    for b in range(B):
        for h in range(H):
            if not pass_mask[b, h]:
                continue
            t = int(t_star[b, h])
            n = nrm[b, t, h]
            if n > 0:
                gz[b, t, h] += gm[b, h] * z[b, t, h] / n
    return np.ascontiguousarray(gz), np.ascontiguousarray(gzq), gv, dgamma


def ska_core_fwd_bwd(z, zq, v, gamma, dy, params: SkaParams = SkaParams(), dtype=np.float64):
    """Convenience: forward then backward; returns ``(y, dz, dzq, dv, dgamma)``."""
    y, cache = ska_core_forward(z, zq, v, gamma, params, dtype)
    dz, dzq, dv, dg = ska_core_backward(dy, cache)
    return y, dz, dzq, dv, dg
