"""Recurrent (decode) inference for one SKA layer on the sm_100a kernels.

Mirrors the SKA part of ``koopman_lm.recurrent`` (upstream
``koopman-lm-fast/koopman_lm/recurrent.py``):

* :class:`SKAState` -- ``SKAState`` (``recurrent.py:48-66``): the fixed-size state
  ``G [B,H,r,r]``, ``M [B,H,r,r]``, ``C_v [B,H,P,r]``, ``z_last [B,H,r]`` (None
  before the first token), ``max_norm [B,1,H,1]`` and ``token_count``, here views
  of one device buffer that the C ABI (``ska_state_*``, ``ska_prefill_state``,
  ``ska_step``) reads and writes;
* :func:`ska_prefill` -- the SKA layer of ``RecurrentKoopmanLM._ska_prefill``
  (``recurrent.py:129-189``): the layer's parallel forward plus the state after
  the prompt, taken from the forward's own chunk statistics (the reference
  recomputes the projections and the statistics a second time);
* :func:`ska_step` -- the SKA layer of ``RecurrentKoopmanLM._ska_step``
  (``recurrent.py:270-375``): one (or several, in order) decode tokens with O(1)
  state.

Both take an :class:`~koopman_mamba_b200.ska.SKAModule` and the layer's input
(after the block's norm) and return the layer's output before the block's
residual, i.e. ``out_proj(eta * y_hat)``.  The standard chunk strategy only, and
``rank <= 32`` for the steps (the kernels' limits); everything runs on the GPU.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ska import _DTYPES, _tensor_desc

__all__ = ["SKAState", "ska_prefill", "ska_step"]


class SKAState:
    """Fixed-size recurrent state of one SKA layer (``recurrent.py:48-66``)."""

    __slots__ = ("buffer", "G", "M", "C_v", "_z_last", "max_norm", "flags", "token_count", "_has_last",
                 "_shape", "_bytes")

    def __init__(self, B, H, r, P, device, dtype=torch.float32, ridge_eps=1e-3):
        if dtype != torch.float32:
            raise TypeError("the SKA state is float32 (as the reference's)")
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("the SKA recurrent state lives on a CUDA (sm_100a) device")
        self._shape = _lib.make_shape(B, 1, H, r, P, 1, 0, ridge_eps)
        self._bytes = _lib.state_size(self._shape)
        self.buffer = torch.empty(self._bytes, dtype=torch.uint8, device=device)
        n = B * H
        off = 0

        def take(count, shape, dt=torch.float32):
            nonlocal off
            t = self.buffer[off:off + count * 4].view(dt).view(*shape)
            off = (off + count * 4 + 255) // 256 * 256
            return t

        self.G = take(n * r * r, (B, H, r, r))
        self.M = take(n * r * r, (B, H, r, r))
        self.C_v = take(n * P * r, (B, H, P, r))
        self._z_last = take(n * r, (B, H, r))
        self.max_norm = take(n, (B, 1, H, 1))
        self.flags = take(n, (B, H), torch.int32)
        self.token_count = 0
        self._has_last = False
        with torch.cuda.device(device):
            _lib.check("ska_state_init", _lib.lib().ska_state_init(
                ctypes.byref(self._shape), ctypes.c_void_p(self.buffer.data_ptr()), self._bytes,
                ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)))

    @property
    def z_last(self):
        return self._z_last if self._has_last else None

    def size_bytes(self, B, H, r, P):
        """Total state size in bytes (float32), as the reference counts it."""
        return B * H * (r * r + r * r + P * r + r + 1) * 4


def _projections(ska, x):
    B, T, _ = x.shape
    r, H, P = ska.rank, ska.H, ska.P
    z = ska.key_proj(x).reshape(B, T, H, r)
    zq = ska.query_proj(x).reshape(B, T, H, r)
    v = ska.value_proj(x).reshape(B, T, H, P)
    dt = z.dtype if z.dtype in _DTYPES else torch.float32
    return [t.to(dt).contiguous() for t in (z, zq, v)]


def _shape(ska, B, T):
    if ska.chunk_strategy != "standard":
        raise NotImplementedError("the recurrent state is defined for chunk_strategy='standard'")
    return _lib.make_shape(B, T, ska.H, ska.rank, ska.P, ska.chunk_size, ska.power_K, ska.ridge_eps)


def _epilogue(ska, y, x):
    B, T = y.shape[:2]
    return ska.out_proj((ska.eta * y.to(x.dtype)).reshape(B, T, ska.H * ska.P))


@torch.no_grad()
def ska_prefill(ska, x):
    """The layer output over the prompt ``x [B, T, d_model]`` and the layer's state
    after it (``recurrent.py:129-189``)."""
    if not x.is_cuda:
        raise RuntimeError("ska_prefill runs on CUDA (sm_100a) devices only")
    B, T, _ = x.shape
    z, zq, v = _projections(ska, x)
    dev = z.device
    shape = _shape(ska, B, T)
    saved_bytes = _lib.forward_workspace_size(shape)   # no backward reads this buffer
    saved = torch.empty(max(saved_bytes, 256), dtype=torch.uint8, device=dev)
    y = torch.empty(B, T, ska.H, ska.P, dtype=z.dtype, device=dev)
    g32 = ska.ssn_gamma.detach().reshape(()).float().contiguous()
    state = SKAState(B, ska.H, ska.rank, ska.P, dev, ridge_eps=ska.ridge_eps)
    io = _DTYPES[z.dtype]
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    dz, dzq, dv, dy = (_tensor_desc(t) for t in (z, zq, v, y))
    L = _lib.lib()
    with torch.cuda.device(dev):
        _lib.check("ska_fwd", L.ska_fwd(ctypes.byref(shape), io, ctypes.byref(dz), ctypes.byref(dzq),
                                        ctypes.byref(dv), ctypes.c_void_p(g32.data_ptr()), ctypes.byref(dy),
                                        ctypes.c_void_p(saved.data_ptr()), saved_bytes, stream))
        _lib.check("ska_prefill_state", L.ska_prefill_state(
            ctypes.byref(shape), io, ctypes.byref(dz), ctypes.byref(dv), ctypes.c_void_p(saved.data_ptr()),
            saved_bytes, ctypes.c_void_p(state.buffer.data_ptr()), state._bytes, stream))
    state.token_count = T
    state._has_last = True
    return _epilogue(ska, y, x), state


@torch.no_grad()
def ska_step(ska, x, state: SKAState):
    """The layer output for the decode tokens ``x [B, T, d_model]`` (usually T = 1),
    one ``_ska_step`` per token in order (``recurrent.py:270-375``); updates
    ``state`` in place."""
    if not x.is_cuda:
        raise RuntimeError("ska_step runs on CUDA (sm_100a) devices only")
    B, T, _ = x.shape
    z, zq, v = _projections(ska, x)
    dev = z.device
    shape = _shape(ska, B, T)
    y = torch.empty(B, T, ska.H, ska.P, dtype=z.dtype, device=dev)
    g32 = ska.ssn_gamma.detach().reshape(()).float().contiguous()
    dz, dzq, dv, dy = (_tensor_desc(t) for t in (z, zq, v, y))
    with torch.cuda.device(dev):
        _lib.check("ska_step", _lib.lib().ska_step(
            ctypes.byref(shape), _DTYPES[z.dtype], ctypes.byref(dz), ctypes.byref(dzq), ctypes.byref(dv),
            ctypes.c_void_p(g32.data_ptr()), ctypes.byref(dy), ctypes.c_void_p(state.buffer.data_ptr()),
            state._bytes, ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
    state.token_count += T
    state._has_last = True
    return _epilogue(ska, y, x)
