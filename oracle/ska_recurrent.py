"""CPU oracle for the SKA recurrent (decode) path: numpy restatement.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module: only
``tests/`` use it, as the checker.  The CUDA library never routes through it.

What it restates (paths relative to the upstream project root, ``KLF`` =
``koopman-lm-fast``):

* ``KLF/koopman_lm/recurrent.py:48-66`` ``SKAState``: the fixed-size state of one
  SKA layer, ``G [B,H,r,r]``, ``M [B,H,r,r]``, ``C_v [B,H,P,r]``, ``z_last [B,H,r]``
  and ``max_norm``;
* ``recurrent.py:129-189`` ``_ska_prefill``: the state after a prompt, from the
  prompt's keys and values normalised by the prompt's max key norm:
  ``G = sum_t z_t z_t^T + ridge I``, ``M = sum_{t>=1} z_t z_{t-1}^T``,
  ``C_v = sum_t v_t z_t^T``, ``z_last = z_{T-1}``;
* ``recurrent.py:270-375`` ``_ska_step``: one token with the max norm frozen at
  its prefill value: rank-1 updates of G, M, C_v, then symmetrise, Cholesky (with
  the 1e-4 jitter on failing slices), ``A_w = M G^{-1}`` spectrally normalised by
  the 6-iteration power iteration (``ska.py:41-58``) and scaled by
  ``clamp(gamma, 1, 1.5)``, ``B_v = C_v G^{-1}``, ``w_q = L^{-1} zq``,
  ``w_f = A_w^K w_q``, ``y = B_v L w_f``.

Parity pin: ``tests/golden/make_golden_recurrent.py`` runs the upstream
``RecurrentKoopmanLM._ska_prefill`` / ``_ska_step`` themselves and stores their
states and outputs; ``tests/test_oracle.py`` checks this restatement against them.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .ska_oracle import _cholesky_solve, _mT, _solve_lower, _spectral_normalize, cholesky_ex

__all__ = ["RecurrentState", "prefill_state", "decode_step"]


@dataclass
class RecurrentState:
    """One SKA layer's recurrent state (``recurrent.py:48-66``); ``z_last`` is
    None before the first token."""

    G: np.ndarray          # [B, H, r, r]
    M: np.ndarray          # [B, H, r, r]
    C: np.ndarray          # [B, H, P, r]
    z_last: np.ndarray | None   # [B, H, r]
    max_norm: np.ndarray   # [B, H]

    def copy(self) -> "RecurrentState":
        return RecurrentState(self.G.copy(), self.M.copy(), self.C.copy(),
                              None if self.z_last is None else self.z_last.copy(), self.max_norm.copy())


def prefill_state(z, v, ridge_eps: float, dtype=np.float64) -> RecurrentState:
    """State after the prompt ``z [B,T,H,r]``, ``v [B,T,H,P]`` (``recurrent.py:150-189``)."""
    z = np.asarray(z, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    B, T, H, r = z.shape
    mx = np.maximum(np.linalg.norm(z, axis=-1).max(axis=1), np.asarray(1e-6, dtype=dtype))   # [B, H]
    zn = z / mx[:, None, :, None]
    G = np.einsum("bthr,bths->bhrs", zn, zn) + np.asarray(ridge_eps, dtype=dtype) * np.eye(r, dtype=dtype)
    M = np.zeros((B, H, r, r), dtype=dtype)
    if T > 1:
        M = np.einsum("bthr,bths->bhrs", zn[:, 1:], zn[:, :-1])
    C = np.einsum("bthp,bthr->bhpr", v, zn)
    return RecurrentState(G, M, C, zn[:, -1].copy(), mx)


def decode_step(state: RecurrentState, z_t, zq_t, v_t, gamma: float, power_K: int,
                power_iters: int = 6, jitter: float = 1e-4) -> np.ndarray:
    """One token (``z_t, zq_t [B,H,r]``, ``v_t [B,H,P]``) through ``_ska_step``
    (``recurrent.py:306-369``).  Updates ``state`` in place and returns ``y_hat``
    ``[B, H, P]`` (before eta and out_proj)."""
    dt = state.G.dtype
    z_t = np.asarray(z_t, dtype=dt)
    zq_t = np.asarray(zq_t, dtype=dt)
    v_t = np.asarray(v_t, dtype=dt)
    B, H, r = z_t.shape
    P = v_t.shape[-1]
    mn = state.max_norm[..., None]
    zn = z_t / mn
    zqn = zq_t / mn
    state.G = state.G + np.einsum("bhr,bhs->bhrs", zn, zn)
    if state.z_last is not None:
        state.M = state.M + np.einsum("bhr,bhs->bhrs", zn, state.z_last)
    state.C = state.C + np.einsum("bhp,bhr->bhpr", v_t, zn)
    state.z_last = zn.copy()

    N = B * H
    G = state.G.reshape(N, r, r)
    M = state.M.reshape(N, r, r)
    C = state.C.reshape(N, P, r)
    Gs = 0.5 * (G + _mT(G))
    L, info = cholesky_ex(Gs)
    Lj, _ = cholesky_ex(Gs + np.asarray(jitter, dtype=dt) * np.eye(r, dtype=dt))
    L = np.where((info > 0)[:, None, None], Lj, L)
    Aw = _mT(_cholesky_solve(_mT(M), L))
    Aw, _, _ = _spectral_normalize(Aw, power_iters)
    Aw = Aw * np.asarray(min(max(gamma, 1.0), 1.5), dtype=dt)
    Bv = _mT(_cholesky_solve(_mT(C), L))
    w = _solve_lower(L, zqn.reshape(N, r, 1))
    for _ in range(power_K):
        w = Aw @ w
    y = Bv @ (L @ w)
    return y.reshape(B, H, P)
