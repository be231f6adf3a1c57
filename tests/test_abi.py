"""CPU: the C-ABI library builds, loads and exports every symbol the header
declares; argument validation runs without touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from koopman_mamba_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "ska_b200.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ska_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_expected_functions():
    assert _declared_functions() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol(built_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", built_lib], check=True, capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\bT (ska_[a-z0-9_]+)$", out, flags=re.M))
    missing = set(_declared_functions()) - exported
    assert not missing, missing
    L = ctypes.CDLL(built_lib)
    for name in _declared_functions():
        assert hasattr(L, name)


def test_abi_version_and_status_strings(built_lib):
    assert _lib.lib().ska_abi_version() == _lib.SKA_ABI_VERSION
    assert _lib.status_string(0) == "ok"
    for code in range(-9, 0):
        assert _lib.status_string(code) != "unknown status"


def _shape(**kw):
    base = dict(B=8, T=2048, H=12, r=32, P=64, chunk_size=64, power_K=2, ridge_eps=1e-3)
    base.update(kw)
    return _lib.make_shape(**base)


def test_workspace_size_config2(built_lib):
    saved, scratch = _lib.workspace_size(_shape())
    n = 8 * 12 * 32                 # B*H*C chunk records
    sw = 2 * 32 * 32 + 64 * 32      # floats per record
    assert saved >= n * sw * 4 and scratch >= n * sw * 4
    assert saved % 256 == 0 and scratch % 256 == 0


@pytest.mark.parametrize("r,P,op_floats", [(32, 64, 6 * 32 * 32), (16, 32, 6 * 32 * 32), (48, 64, 6 * 64 * 64),
                                            (64, 64, 6 * 64 * 64), (48, 96, 0), (36, 64, 0),
                                            (40, 64, 6 * 64 * 64)])
def test_forward_workspace_is_the_leading_part(built_lib, r, P, op_floats):
    # the chunk operators the backward reads sit at the end of the saved buffer: a
    # forward with no backward after it needs only what comes before them
    s = _shape(r=r, P=P)
    saved, _ = _lib.workspace_size(s)
    fwd = _lib.forward_workspace_size(s)
    n = 8 * 12 * 32
    assert fwd % 256 == 0 and fwd >= n * (2 * r * r + P * r) * 4
    assert saved - fwd == -(-(n * op_floats * 4) // 256) * 256
    # the factor kernels' Li (r <= 32: Li^T, 4 KB per chunk; the four-warp shapes:
    # three 4 KB tiles) is part of the forward's share, with the W/m planes
    lis = 1024 if r <= 32 else (3 * 1024 if op_floats else 0)
    assert fwd >= n * (2 * r * r + P * r + P * r + lis) * 4


@pytest.mark.parametrize("kw,code", [
    (dict(T=0), -2), (dict(H=0), -2), (dict(r=0), -2), (dict(B=-1), -2), (dict(power_K=-1), -2),
    (dict(chunk_size=0), -2), (dict(r=65), -3), (dict(P=129), -3), (dict(chunk_size=257), -3),
    (dict(power_K=9), -3), (dict(strategy=7), -8),
])
def test_shape_validation(built_lib, kw, code):
    with pytest.raises(_lib.SkaError) as ei:
        _lib.workspace_size(_shape(**kw))
    assert ei.value.code == code


def test_fwd_validation_before_any_cuda_call(built_lib):
    L = _lib.lib()
    s = _shape(B=1, T=64, H=1)
    t = _lib.SkaTensor(0, 0, 0, 0)
    # null data pointers with work to do
    rc = L.ska_fwd(ctypes.byref(s), 1, ctypes.byref(t), ctypes.byref(t), ctypes.byref(t), None,
                   ctypes.byref(t), None, 0, None)
    assert rc == -1
    # unknown dtype
    rc = L.ska_fwd(ctypes.byref(s), 5, ctypes.byref(t), ctypes.byref(t), ctypes.byref(t), None,
                   ctypes.byref(t), None, 0, None)
    assert rc == -4
    # misaligned bf16 pointer
    bad = _lib.SkaTensor(0x1001, 0, 0, 0)
    rc = L.ska_fwd(ctypes.byref(s), 1, ctypes.byref(bad), ctypes.byref(bad), ctypes.byref(bad), None,
                   ctypes.byref(bad), None, 0, None)
    assert rc == -6
    # B == 0 is a no-op
    s0 = _shape(B=0)
    rc = L.ska_fwd(ctypes.byref(s0), 1, ctypes.byref(t), ctypes.byref(t), ctypes.byref(t), None,
                   ctypes.byref(t), None, 0, None)
    assert rc == 0
    # workspace too small
    ok = _lib.SkaTensor(0x1000, 0, 0, 0)
    rc = L.ska_fwd(ctypes.byref(s), 1, ctypes.byref(ok), ctypes.byref(ok), ctypes.byref(ok),
                   ctypes.c_void_p(0x2000), ctypes.byref(ok), ctypes.c_void_p(0x10000), 16, None)
    assert rc == -5


TC = _lib.SKA_PATH_TC_STATS | _lib.SKA_PATH_TC_TOKEN_BWD
RD = _lib.SKA_PATH_TC_READOUT_FWD
OPS = _lib.SKA_PATH_TC_CHUNK_FWD | _lib.SKA_PATH_TC_CHUNK_BWD   # r <= 32 chunk operators on tcgen05


def _contig(base, B, T, H, D):
    return _lib.SkaTensor(base, T * H * D, H * D, D)


@pytest.mark.parametrize("kw,dtype,zt,want", [
    # config 2 in bf16, contiguous: every tensor-core kernel (chunk operators four per
    # CTA on tcgen05), statistics and scan fused (96 series)
    (dict(), 1, None, TC | _lib.SKA_PATH_WARP_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD | _lib.SKA_PATH_FUSED_SCAN | RD | OPS),
    # too few series to occupy the SMs one CTA per series: statistics and scan apart
    (dict(B=2, H=4), 1, None, TC | _lib.SKA_PATH_WARP_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD | RD | OPS),
    # fp32 tensors: CUDA-core token kernels
    (dict(), 0, None, _lib.SKA_PATH_WARP_CHUNK),
    # r = 64 (config 3): tensor-core token kernels, readout and readout gradient,
    # four-warp chunk operators forward and backward
    (dict(r=64, chunk_size=128), 1, None,
     TC | RD | _lib.SKA_PATH_QUAD_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD | _lib.SKA_PATH_QUAD_CHUNK_BWD),
    # r = 48 (the module default): the same
    (dict(r=48), 1, None,
     TC | RD | _lib.SKA_PATH_QUAD_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD | _lib.SKA_PATH_QUAD_CHUNK_BWD),
    # power_K = 3 at r = 48: the backward's one-CTA operator kernel recomputes the forward
    (dict(r=48, power_K=3), 1, None, TC | RD | _lib.SKA_PATH_QUAD_CHUNK),
    # chunk 256: tensor-core statistics only
    (dict(r=64, chunk_size=256), 1, None, _lib.SKA_PATH_TC_STATS),
    # P % 16 != 0: tensor-core statistics only
    (dict(P=40), 1, None, _lib.SKA_PATH_TC_STATS | _lib.SKA_PATH_WARP_CHUNK | _lib.SKA_PATH_FUSED_SCAN),
    # r = 16 (config 5): every tensor-core kernel but the fused statistics + scan
    (dict(r=16), 1, None, TC | _lib.SKA_PATH_WARP_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD | RD | OPS),
    # r = 16, P = 32 (config 5's head): the same
    (dict(r=16, P=32), 1, None, TC | _lib.SKA_PATH_WARP_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD | RD | OPS),
    # token stride not a multiple of 16 bytes: CUDA-core token kernels
    (dict(), 1, _lib.SkaTensor(0x1000, 2048 * 12 * 36, 12 * 36, 36), _lib.SKA_PATH_WARP_CHUNK),
    # decay strategy shares the token kernels and the fused statistics + scan
    (dict(strategy=_lib.SKA_STRATEGY_DECAY, decay_alpha=0.9), 1, None,
     TC | _lib.SKA_PATH_WARP_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD | _lib.SKA_PATH_FUSED_SCAN | RD | OPS),
])
def test_kernel_path_selection(built_lib, kw, dtype, zt, want):
    s = _shape(**kw)
    z = zt or _contig(0x1000, s.B, s.T, s.H, s.r)
    v = _contig(0x100000, s.B, s.T, s.H, s.P)
    assert _lib.lib().ska_kernel_path(ctypes.byref(s), dtype, ctypes.byref(z), ctypes.byref(v)) == want


def test_kernel_path_rejects_what_ska_fwd_rejects(built_lib):
    L = _lib.lib()
    s = _shape()
    t = _lib.SkaTensor(0, 0, 0, 0)
    assert L.ska_kernel_path(ctypes.byref(s), 1, ctypes.byref(t), ctypes.byref(t)) == -1
    assert L.ska_kernel_path(ctypes.byref(s), 9, ctypes.byref(t), ctypes.byref(t)) == -4
