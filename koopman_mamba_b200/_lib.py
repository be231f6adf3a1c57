"""ctypes binding of ``libska_b200.so`` (the C ABI declared in ``include/ska_b200.h``).

The library is the only compute path: if it is missing or cannot be loaded the
import of :func:`lib` raises, and nothing falls back to another implementation.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libska_b200.so")

SKA_ABI_VERSION = 1
SKA_DTYPE_F32 = 0
SKA_DTYPE_BF16 = 1
SKA_DTYPE_BF16_Y32 = 2
SKA_STRATEGY_STANDARD = 0
SKA_STRATEGY_DECAY = 1

# Functions declared in include/ska_b200.h (checked against the header by the tests).
EXPORTED = (
    "ska_abi_version",
    "ska_status_string",
    "ska_workspace_size",
    "ska_forward_workspace_size",
    "ska_fwd",
    "ska_bwd",
    "ska_set_profile_events",
    "ska_fwd_noalloc",
    "ska_kernel_path",
    "ska_set_wait_limit",
    "ska_check_status",
    "ska_state_size",
    "ska_state_init",
    "ska_prefill_state",
    "ska_step",
)
SKA_ERR_NULL = -1
SKA_ERR_SHAPE = -2
SKA_ERR_UNSUPPORTED = -3
SKA_ERR_DTYPE = -4
SKA_ERR_WORKSPACE = -5
SKA_ERR_ALIGN = -6
SKA_ERR_LAUNCH = -7
SKA_ERR_STRATEGY = -8
SKA_ERR_TIMEOUT = -9
SKA_STATUS_BWD_BASE = 16
SKA_WAIT_LIMIT_DEFAULT = 0xFFFFFFFF
SKA_PATH_TC_STATS = 1
SKA_PATH_WARP_CHUNK = 2
SKA_PATH_TC_TOKEN_BWD = 4
SKA_PATH_TC_READOUT_BWD = 8
SKA_PATH_FUSED_SCAN = 16
SKA_PATH_TC_READOUT_FWD = 32
SKA_PATH_QUAD_CHUNK = 64
SKA_PATH_TC_CHUNK_FWD = 128
SKA_PATH_TC_CHUNK_BWD = 256
SKA_PATH_QUAD_CHUNK_BWD = 512
SKA_NOALLOC_SCRATCH_BYTES = 16 << 20
SKA_PROFILE_EVENTS = 10


class SkaShape(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int64),
        ("T", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("r", ctypes.c_int64),
        ("P", ctypes.c_int64),
        ("chunk_size", ctypes.c_int64),
        ("power_K", ctypes.c_int32),
        ("strategy", ctypes.c_int32),
        ("ridge_eps", ctypes.c_float),
        ("decay_alpha", ctypes.c_float),
    ]


class SkaTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("stride_b", ctypes.c_int64),
        ("stride_t", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
    ]


class SkaError(RuntimeError):
    """A non-zero status returned by the SKA C ABI."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def _declare(L: ctypes.CDLL) -> None:
    P = ctypes.POINTER
    L.ska_abi_version.argtypes = []
    L.ska_abi_version.restype = ctypes.c_int
    L.ska_status_string.argtypes = [ctypes.c_int]
    L.ska_status_string.restype = ctypes.c_char_p
    L.ska_workspace_size.argtypes = [P(SkaShape), P(ctypes.c_size_t), P(ctypes.c_size_t)]
    L.ska_workspace_size.restype = ctypes.c_int
    L.ska_forward_workspace_size.argtypes = [P(SkaShape), P(ctypes.c_size_t)]
    L.ska_forward_workspace_size.restype = ctypes.c_int
    L.ska_fwd.argtypes = [P(SkaShape), ctypes.c_int, P(SkaTensor), P(SkaTensor), P(SkaTensor),
                          ctypes.c_void_p, P(SkaTensor), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.ska_fwd.restype = ctypes.c_int
    L.ska_bwd.argtypes = [P(SkaShape), ctypes.c_int, P(SkaTensor), P(SkaTensor), P(SkaTensor),
                          ctypes.c_void_p, P(SkaTensor), ctypes.c_void_p, ctypes.c_size_t,
                          ctypes.c_void_p, ctypes.c_size_t, P(SkaTensor), P(SkaTensor), P(SkaTensor),
                          ctypes.c_void_p, ctypes.c_void_p]
    L.ska_bwd.restype = ctypes.c_int
    L.ska_set_profile_events.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]
    L.ska_set_profile_events.restype = ctypes.c_int
    L.ska_kernel_path.argtypes = [P(SkaShape), ctypes.c_int, P(SkaTensor), P(SkaTensor)]
    L.ska_kernel_path.restype = ctypes.c_int
    L.ska_fwd_noalloc.argtypes = [P(SkaShape), ctypes.c_int, P(SkaTensor), P(SkaTensor), P(SkaTensor),
                                  ctypes.c_void_p, P(SkaTensor), ctypes.c_void_p]
    L.ska_fwd_noalloc.restype = ctypes.c_int
    L.ska_set_wait_limit.argtypes = [ctypes.c_uint32]
    L.ska_set_wait_limit.restype = ctypes.c_int
    L.ska_check_status.argtypes = [P(SkaShape), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                   ctypes.c_void_p, P(ctypes.c_int64), P(ctypes.c_int)]
    L.ska_check_status.restype = ctypes.c_int
    L.ska_state_size.argtypes = [P(SkaShape), P(ctypes.c_size_t)]
    L.ska_state_size.restype = ctypes.c_int
    L.ska_state_init.argtypes = [P(SkaShape), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.ska_state_init.restype = ctypes.c_int
    L.ska_prefill_state.argtypes = [P(SkaShape), ctypes.c_int, P(SkaTensor), P(SkaTensor), ctypes.c_void_p,
                                    ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.ska_prefill_state.restype = ctypes.c_int
    L.ska_step.argtypes = [P(SkaShape), ctypes.c_int, P(SkaTensor), P(SkaTensor), P(SkaTensor), ctypes.c_void_p,
                           P(SkaTensor), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.ska_step.restype = ctypes.c_int


def lib() -> ctypes.CDLL:
    """Load (once) and return the SKA library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m koopman_mamba_b200.build` "
                    "(there is no non-CUDA implementation of the SKA core)")
            L = ctypes.CDLL(LIB_PATH)
            _declare(L)
            v = L.ska_abi_version()
            if v != SKA_ABI_VERSION:
                raise RuntimeError(f"libska_b200 ABI version {v}, expected {SKA_ABI_VERSION}")
            _lib = L
    return _lib


def status_string(code: int) -> str:
    return lib().ska_status_string(int(code)).decode()


def check(fn: str, code: int) -> None:
    if code != 0:
        raise SkaError(fn, code, status_string(code))


def make_shape(B, T, H, r, P, chunk_size, power_K, ridge_eps, strategy=SKA_STRATEGY_STANDARD,
               decay_alpha=1.0) -> SkaShape:
    return SkaShape(int(B), int(T), int(H), int(r), int(P), int(chunk_size), int(power_K),
                    int(strategy), float(ridge_eps), float(decay_alpha))


def state_size(shape: SkaShape) -> int:
    n = ctypes.c_size_t(0)
    check("ska_state_size", lib().ska_state_size(ctypes.byref(shape), ctypes.byref(n)))
    return int(n.value)


def forward_workspace_size(shape: SkaShape) -> int:
    """Saved-buffer bytes for a forward that no backward follows."""
    n = ctypes.c_size_t(0)
    check("ska_forward_workspace_size", lib().ska_forward_workspace_size(ctypes.byref(shape), ctypes.byref(n)))
    return int(n.value)


def workspace_size(shape: SkaShape) -> tuple[int, int]:
    saved = ctypes.c_size_t(0)
    scratch = ctypes.c_size_t(0)
    check("ska_workspace_size", lib().ska_workspace_size(ctypes.byref(shape), ctypes.byref(saved),
                                                         ctypes.byref(scratch)))
    return int(saved.value), int(scratch.value)
