"""GPU: ska_fwd_noalloc, the forward for callers that cannot allocate.

Some callers cannot call cudaMalloc: FFI hosts that have no CUDA allocator of
their own, and inference loops that must not allocate between launches.  For
them the library exports ska_fwd_noalloc, whose workspace is a fixed device
array compiled into the library (SKA_NOALLOC_SCRATCH_BYTES).  This file checks,
through the C ABI, that it returns what ska_fwd returns for the same inputs, on
two calls in a row (the shared array keeps the first call's contents), and that
a problem larger than the array is refused.  It is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

from koopman_mamba_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 1e-4   # the fp32 parity bar; the two paths run the same kernels


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _desc(t):
    return _lib.SkaTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _inputs(B, T, H, r, P, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(64)
    return [(torch.randn(B, T, H, n, generator=g) * s).to(DEV, dtype) for n in (r, r, P)]


def _fwd_both(B, T, H, r, P, seed, dtype, chunk=64):
    L = _lib.lib()
    z, zq, v = _inputs(B, T, H, r, P, seed, dtype)
    gamma = torch.tensor(1.1, device=DEV, dtype=torch.float32)
    shape = _lib.make_shape(B, T, H, r, P, chunk, 2, 1e-3)
    saved_bytes, _ = _lib.workspace_size(shape)
    assert saved_bytes <= _lib.SKA_NOALLOC_SCRATCH_BYTES
    saved = torch.empty(saved_bytes, dtype=torch.uint8, device=DEV)
    y_ref = torch.empty(B, T, H, P, dtype=dtype, device=DEV)
    y_new = torch.full((B, T, H, P), float("nan"), dtype=dtype, device=DEV)
    io = _lib.SKA_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.SKA_DTYPE_F32
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    dz, dzq, dv, dyr, dyn = (_desc(t) for t in (z, zq, v, y_ref, y_new))
    gp = ctypes.c_void_p(gamma.data_ptr())
    _lib.check("ska_fwd", L.ska_fwd(ctypes.byref(shape), io, ctypes.byref(dz), ctypes.byref(dzq), ctypes.byref(dv),
                                    gp, ctypes.byref(dyr), ctypes.c_void_p(saved.data_ptr()), saved_bytes, stream))
    _lib.check("ska_fwd_noalloc", L.ska_fwd_noalloc(ctypes.byref(shape), io, ctypes.byref(dz), ctypes.byref(dzq),
                                                    ctypes.byref(dv), gp, ctypes.byref(dyn), stream))
    torch.cuda.synchronize()
    return y_ref.double(), y_new.double()


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_noalloc_matches_ska_fwd_two_calls_in_a_row():
    # first call: config-1 shape in fp32; second call: another shape in bf16,
    # reusing the array that still holds the first call's workspace
    y_ref, y_new = _fwd_both(2, 512, 4, 16, 64, 0, torch.float32)
    assert torch.isfinite(y_new).all()
    assert _rel(y_new, y_ref) <= TOL
    y_ref, y_new = _fwd_both(1, 600, 3, 32, 64, 7, torch.bfloat16)
    assert torch.isfinite(y_new).all()
    assert _rel(y_new, y_ref) <= TOL


def test_noalloc_refuses_problems_larger_than_its_array():
    L = _lib.lib()
    shape = _lib.make_shape(8, 2048, 12, 32, 64, 64, 2, 1e-3)   # needs ~50 MB of workspace
    saved_bytes = _lib.forward_workspace_size(shape)
    assert saved_bytes > _lib.SKA_NOALLOC_SCRATCH_BYTES
    t = _lib.SkaTensor(0, 0, 0, 0)
    rc = L.ska_fwd_noalloc(ctypes.byref(shape), _lib.SKA_DTYPE_BF16, ctypes.byref(t), ctypes.byref(t),
                           ctypes.byref(t), None, ctypes.byref(t), None)
    assert rc == -5   # SKA_ERR_WORKSPACE, nothing launched
