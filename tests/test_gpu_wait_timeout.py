"""GPU: the bounded waits of the tensor-core kernels expire without a fault.

Every mbarrier wait in the TMA + tcgen05 kernels gives up after a bounded number
of polls.  ska_set_wait_limit(0) makes the first wait of every role give up at
once (a wait on a flag that nothing sets, made deterministic), while the waits
that drain the copies and products already in flight keep the full limit.  The
launch must then complete, record the expiry in the status entries that
ska_check_status reads (the drop-in contract's "scan-wait timeout" error), write
NaN into the affected outputs, and leave the context usable: a run with the
default limit right afterwards gives the clean result bit for bit.
"""
import ctypes
import math

import pytest
import torch

from koopman_mamba_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(autouse=True)
def _restore_limit():
    yield
    _lib.lib().ska_set_wait_limit(_lib.SKA_WAIT_LIMIT_DEFAULT)


def _desc(t):
    return _lib.SkaTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


class _Problem:
    """bf16 inputs laid out for the tensor-core kernels, with caller-owned buffers."""

    def __init__(self, B, T, H, r=32, P=64, chunk=64, seed=3):
        g = torch.Generator().manual_seed(seed)
        s = 1.0 / math.sqrt(64)
        self.z, self.zq, self.v = ((torch.randn(B, T, H, n, generator=g) * s).to(DEV, torch.bfloat16)
                                   for n in (r, r, P))
        self.dy = torch.randn(B, T, H, P, generator=g).to(DEV, torch.bfloat16)
        self.shape = _lib.make_shape(B, T, H, r, P, chunk, 2, 1e-3)
        self.saved_bytes, self.scratch_bytes = _lib.workspace_size(self.shape)
        self.saved = torch.empty(self.saved_bytes, dtype=torch.uint8, device=DEV)
        self.scratch = torch.empty(self.scratch_bytes, dtype=torch.uint8, device=DEV)
        self.gamma = torch.tensor(1.1, device=DEV)
        self.dgamma = torch.empty((), device=DEV)
        self.y = torch.empty(B, T, H, P, dtype=torch.bfloat16, device=DEV)
        self.dz, self.dzq, self.dv = (torch.empty_like(t) for t in (self.z, self.zq, self.v))
        self.stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
        self.L = _lib.lib()

    def path(self):
        return self.L.ska_kernel_path(ctypes.byref(self.shape), _lib.SKA_DTYPE_BF16, ctypes.byref(_desc(self.z)),
                                      ctypes.byref(_desc(self.v)))

    def fwd(self):
        d = [_desc(t) for t in (self.z, self.zq, self.v, self.y)]
        _lib.check("ska_fwd", self.L.ska_fwd(ctypes.byref(self.shape), _lib.SKA_DTYPE_BF16, *map(ctypes.byref, d[:3]),
                                             ctypes.c_void_p(self.gamma.data_ptr()), ctypes.byref(d[3]),
                                             ctypes.c_void_p(self.saved.data_ptr()), self.saved_bytes, self.stream))

    def bwd(self):
        d = [_desc(t) for t in (self.z, self.zq, self.v, self.dy, self.dz, self.dzq, self.dv)]
        rc = self.L.ska_bwd(ctypes.byref(self.shape), _lib.SKA_DTYPE_BF16, *map(ctypes.byref, d[:3]),
                            ctypes.c_void_p(self.gamma.data_ptr()), ctypes.byref(d[3]),
                            ctypes.c_void_p(self.saved.data_ptr()), self.saved_bytes,
                            ctypes.c_void_p(self.scratch.data_ptr()), self.scratch_bytes,
                            *map(ctypes.byref, d[4:]), ctypes.c_void_p(self.dgamma.data_ptr()), self.stream)
        _lib.check("ska_bwd", rc)

    def status(self, fwd=True, bwd=True):
        bad, code = ctypes.c_int64(0), ctypes.c_int(0)
        rc = self.L.ska_check_status(ctypes.byref(self.shape),
                                     ctypes.c_void_p(self.saved.data_ptr()) if fwd else None, self.saved_bytes,
                                     ctypes.c_void_p(self.scratch.data_ptr()) if bwd else None, self.scratch_bytes,
                                     self.stream, ctypes.byref(bad), ctypes.byref(code))
        return rc, bad.value, code.value


@pytest.mark.parametrize("B,H", [(4, 16), (1, 3)])
def test_forward_wait_expiry_is_reported_and_recoverable(B, H):
    """(4, 16): 64 series, the fused statistics + scan kernel; (1, 3): the
    one-chunk-per-CTA statistics kernel."""
    p = _Problem(B, 256, H)
    assert p.path() & _lib.SKA_PATH_TC_STATS
    fused = bool(p.path() & _lib.SKA_PATH_FUSED_SCAN)
    assert fused == (B * H >= 64)
    p.fwd()
    assert p.status(bwd=False) == (0, -1, 0)
    clean = p.y.clone()
    assert torch.isfinite(clean.float()).all()

    p.L.ska_set_wait_limit(0)
    p.y.zero_()
    p.fwd()
    rc, bad, code = p.status(bwd=False)
    assert rc == _lib.SKA_ERR_TIMEOUT
    # bits 0-1: the statistics kernel, bits 2-3: the tensor-core readout kernel,
    # bits 4-5: the tensor-core chunk-operator kernel (a product wait: 2)
    assert bad == 0 and (code & 3) in (1, 2) and ((code >> 2) & 3) in (0, 1, 2)
    assert (code >> 4) == (2 if p.path() & _lib.SKA_PATH_TC_CHUNK_FWD else 0)
    assert torch.isnan(p.y.float()).any()

    p.L.ska_set_wait_limit(_lib.SKA_WAIT_LIMIT_DEFAULT)
    p.fwd()
    assert p.status(bwd=False) == (0, -1, 0)
    assert torch.equal(p.y, clean)


def test_backward_wait_expiry_is_reported_and_recoverable():
    p = _Problem(4, 256, 16)
    want = _lib.SKA_PATH_TC_TOKEN_BWD | _lib.SKA_PATH_TC_READOUT_BWD
    assert p.path() & want == want
    p.fwd()
    p.bwd()
    assert p.status() == (0, -1, 0)
    clean = [t.clone() for t in (p.dz, p.dzq, p.dv)]
    assert all(torch.isfinite(t.float()).all() for t in clean)

    p.L.ska_set_wait_limit(0)
    p.bwd()
    rc, bad, code = p.status()
    assert rc == _lib.SKA_ERR_TIMEOUT
    assert bad == 0 and code > _lib.SKA_STATUS_BWD_BASE
    # bits 4-5: the tensor-core chunk-operator kernel (a product wait: 2)
    assert ((code - _lib.SKA_STATUS_BWD_BASE) >> 4) == (2 if p.path() & _lib.SKA_PATH_TC_CHUNK_BWD else 0)
    for t in (p.dz, p.dzq, p.dv):
        assert torch.isnan(t.float()).any()

    p.L.ska_set_wait_limit(_lib.SKA_WAIT_LIMIT_DEFAULT)
    p.bwd()
    assert p.status() == (0, -1, 0)
    for a, b in zip((p.dz, p.dzq, p.dv), clean):
        assert torch.equal(a, b)
