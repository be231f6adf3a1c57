"""GPU parity: the sm_100a SKA core (through the C ABI) against the oracle and
the reference's golden vectors.

Tolerances (relative Frobenius norm, the parity bar of the spec):
  * fp32 I/O: 1e-4 on y, dz, dzq, dv;  dgamma within 2e-4 * max(1, |ref|)
  * bf16 I/O: 2e-2 on y, dz, dzq, dv and dgamma, against the oracle fed the
    same bf16-rounded inputs (upcast to fp32, as ska.py:436-438 does).
"""
import math

import numpy as np
import pytest
import torch

from koopman_mamba_b200 import SKAModule, ska_core
from koopman_mamba_b200._lib import SkaError
from oracle.ska_oracle import SkaParams, rel_fro, ska_core_forward, ska_core_fwd_bwd
from tests._golden import core_cases, load, params_of, strategy_kwargs

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_TOL = 2e-2
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def run_cuda(z, zq, v, gamma, dy, dtype, **kw):
    """Forward + backward through the C ABI; returns numpy float64 results."""
    t = [torch.as_tensor(np.ascontiguousarray(a)).to(DEV, dtype).requires_grad_(True) for a in (z, zq, v)]
    g = torch.tensor(float(gamma), device=DEV, requires_grad=True)
    y = ska_core(*t, g, **kw)
    out = [y.detach()]
    if dy is not None:
        y.backward(torch.as_tensor(np.ascontiguousarray(dy)).to(DEV, dtype))
        out += [t[0].grad, t[1].grad, t[2].grad, g.grad]
    torch.cuda.synchronize()
    return [o.double().cpu().numpy() if o.dim() else float(o) for o in out]


def bf16_round(a):
    return torch.as_tensor(np.ascontiguousarray(a)).bfloat16().float().numpy()


def assert_close(got, ref, tol, names=("y", "dz", "dzq", "dv")):
    for g, r, n in zip(got, ref, names):
        e = rel_fro(g, r)
        assert e <= tol, f"{n}: rel err {e:.3e} > {tol:.1e}"


@pytest.mark.parametrize("case", core_cases())
def test_golden_fp32(case):
    d = load(case)
    y, dz, dzq, dv, dg = run_cuda(d["z"], d["zq"], d["v"], d["meta_gamma"], d["dy"], torch.float32,
                                  **strategy_kwargs(d))
    assert_close((y, dz, dzq, dv), (d["y_f64"], d["dz_f64"], d["dzq_f64"], d["dv_f64"]), FP32_TOL)
    ref = float(d["dgamma_f64"])
    assert abs(dg - ref) <= 2e-4 * max(1.0, abs(ref)), (dg, ref)


@pytest.mark.parametrize("case", core_cases())
def test_golden_bf16_io(case):
    d = load(case)
    z, zq, v, dy = (bf16_round(d[k]) for k in ("z", "zq", "v", "dy"))
    y, dz, dzq, dv, dg = run_cuda(z, zq, v, d["meta_gamma"], dy, torch.bfloat16, **strategy_kwargs(d))
    ry, rdz, rdzq, rdv, rdg = ska_core_fwd_bwd(z, zq, v, float(d["meta_gamma"]), dy, params_of(d))
    assert_close((y, dz, dzq, dv), (ry, rdz, rdzq, rdv), BF16_TOL)
    assert abs(dg - rdg) <= BF16_TOL * max(1.0, abs(rdg))


def _inputs(B, T, H, r, P, seed, bf16=True, dy=True):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(64)
    out = [torch.randn(B, T, H, r, generator=g) * s, torch.randn(B, T, H, r, generator=g) * s,
           torch.randn(B, T, H, P, generator=g) * s]
    if dy:
        out.append(torch.randn(B, T, H, P, generator=g))
    if bf16:
        out = [t.bfloat16().float() for t in out]
    return [t.numpy() for t in out]


def test_config1_fp32():
    """Config 1: B=2 H=4 L=512 d=64 r=16, ridge 1e-3, chunk 64, seed 0, fp32."""
    z, zq, v, dy = _inputs(2, 512, 4, 16, 64, 0, bf16=False)
    got = run_cuda(z, zq, v, 1.0, dy, torch.float32)
    ref = ska_core_fwd_bwd(z, zq, v, 1.0, dy, SkaParams())
    assert_close(got[:4], ref[:4], FP32_TOL)
    assert abs(got[4] - ref[4]) <= 2e-4 * max(1.0, abs(ref[4]))


def test_config2_bf16_full_size():
    """Config 2: B=8 H=12 L=2048 d=64 r=32, ridge 1e-3, chunk 64, seed 1, bf16 I/O, fwd+bwd."""
    z, zq, v, dy = _inputs(8, 2048, 12, 32, 64, 1)
    got = run_cuda(z, zq, v, 1.0, dy, torch.bfloat16)
    ref = ska_core_fwd_bwd(z, zq, v, 1.0, dy, SkaParams())
    assert_close(got[:4], ref[:4], BF16_TOL)
    assert abs(got[4] - ref[4]) <= BF16_TOL * max(1.0, abs(ref[4]))


def _oracle_heads_forward(args):
    z, zq, v, chunk = args
    return ska_core_forward(z, zq, v, 1.0, SkaParams(chunk_size=chunk), np.float32)[0]


def test_config3_bf16_forward_all_heads():
    """Config 3 (B=1 H=16 L=32768 r=64 chunk 128, seed 2) forward, every head at full
    length against the oracle, head by head (the four-warp chunk operators and the
    tensor-core readout)."""
    from koopman_mamba_b200 import _lib
    zt = torch.empty(1, 32768, 16, 64, dtype=torch.bfloat16, device=DEV)
    assert _path(zt, zt, 64, 64, chunk=128) & _lib.SKA_PATH_QUAD_CHUNK
    z, zq, v = _inputs(1, 32768, 16, 64, 64, 2, dy=False)
    (y,) = run_cuda(z, zq, v, 1.0, None, torch.bfloat16, chunk_size=128)
    assert np.all(np.isfinite(y))
    refs = [_oracle_heads_forward((z[:, :, h:h + 1], zq[:, :, h:h + 1], v[:, :, h:h + 1], 128)) for h in range(16)]
    ref = np.concatenate(refs, axis=2)
    assert rel_fro(y, ref) <= BF16_TOL
    for h in range(16):
        assert rel_fro(y[:, :, h], ref[:, :, h]) <= BF16_TOL, h


def test_config3_bf16_backward_full_size():
    """Config 3 shape forward + backward through the C ABI (all 16 heads, L=32768,
    r=64, chunk 128), checked against the oracle on 3 heads at full length (the
    series are independent; the backward runs the four-warp chunk operators from
    the operators the forward kept)."""
    from koopman_mamba_b200 import _lib
    zt = torch.empty(1, 32768, 16, 64, dtype=torch.bfloat16, device=DEV)
    assert _path(zt, zt, 64, 64, chunk=128) & _lib.SKA_PATH_QUAD_CHUNK_BWD
    z, zq, v, dy = _inputs(1, 32768, 16, 64, 64, 2)
    got = run_cuda(z, zq, v, 1.0, dy, torch.bfloat16, chunk_size=128)
    heads = [0, 9, 15]
    sub = [a[:, :, heads] for a in (z, zq, v, dy)]
    ref = ska_core_fwd_bwd(*sub[:3], 1.0, sub[3], SkaParams(chunk_size=128), np.float32)
    for g, r_, n in zip(got[:4], ref[:4], ("y", "dz", "dzq", "dv")):
        assert rel_fro(g[:, :, heads], r_) <= BF16_TOL, n
    assert all(np.all(np.isfinite(g)) for g in got[:4])


def test_fused_projection_strides_bitwise():
    """z, zq, v as column slices of one fused projection output (the ska_fast layout)."""
    B, T, H, r, P = 2, 300, 3, 16, 32
    g = torch.Generator().manual_seed(5)
    fused = (torch.randn(B, T, 2 * H * r + H * P, generator=g) / 8).to(DEV, torch.bfloat16)
    z = fused[:, :, :H * r].reshape(B, T, H, r)
    zq = fused[:, :, H * r:2 * H * r].reshape(B, T, H, r)
    v = fused[:, :, 2 * H * r:].reshape(B, T, H, P)
    gm = torch.tensor(1.1, device=DEV)
    y1 = ska_core(z, zq, v, gm)
    y2 = ska_core(z.contiguous(), zq.contiguous(), v.contiguous(), gm)
    assert torch.equal(y1, y2)


def _path(z, v, r, P, chunk=64, power_K=2):
    from koopman_mamba_b200 import _lib
    import ctypes
    B, T, H = z.shape[0], z.shape[1], z.shape[2]
    s = _lib.make_shape(B, T, H, r, P, chunk, power_K, 1e-3)
    tz = _lib.SkaTensor(z.data_ptr(), z.stride(0), z.stride(1), z.stride(2))
    tv = _lib.SkaTensor(v.data_ptr(), v.stride(0), v.stride(1), v.stride(2))
    return _lib.lib().ska_kernel_path(ctypes.byref(s), _lib.SKA_DTYPE_BF16, ctypes.byref(tz), ctypes.byref(tv))


def test_fused_projection_strides_tensor_core_stats():
    """r = 32 slices of one fused projection: strided TMA tiles give the bits of the
    contiguous layout, and both take the TMA + tcgen05 statistics kernel."""
    from koopman_mamba_b200 import _lib
    B, T, H, r, P = 2, 333, 3, 32, 64
    g = torch.Generator().manual_seed(6)
    fused = (torch.randn(B, T, 2 * H * r + H * P, generator=g) / 8).to(DEV, torch.bfloat16)
    z = fused[:, :, :H * r].reshape(B, T, H, r)
    zq = fused[:, :, H * r:2 * H * r].reshape(B, T, H, r)
    v = fused[:, :, 2 * H * r:].reshape(B, T, H, P)
    tc = _lib.SKA_PATH_TC_STATS | _lib.SKA_PATH_TC_TOKEN_BWD | _lib.SKA_PATH_TC_READOUT_BWD
    assert _path(z, v, r, P) & tc == tc
    assert _path(z.contiguous(), v.contiguous(), r, P) & tc == tc
    dy = (torch.randn(B, T, H, P, generator=g)).to(DEV, torch.bfloat16)
    outs = []
    for views in ((z, zq, v), (z.contiguous(), zq.contiguous(), v.contiguous())):
        leaves = [t.detach().requires_grad_(True) for t in views]
        gm = torch.tensor(1.1, device=DEV, requires_grad=True)
        y = ska_core(*leaves, gm)
        y.backward(dy)
        outs.append([y.detach()] + [t.grad for t in leaves] + [gm.grad])
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    np_in = [t.float().cpu().numpy() for t in (z, zq, v)]
    ref = ska_core_fwd_bwd(*np_in, 1.1, dy.float().cpu().numpy(), SkaParams())
    got = [t.double().cpu().numpy() for t in outs[0][:4]]
    assert_close(got, ref[:4], BF16_TOL)


def test_config2_takes_the_tensor_core_statistics_kernel():
    from koopman_mamba_b200 import _lib
    z = torch.empty(8, 2048, 12, 32, dtype=torch.bfloat16, device=DEV)
    v = torch.empty(8, 2048, 12, 64, dtype=torch.bfloat16, device=DEV)
    assert _path(z, v, 32, 64) == (_lib.SKA_PATH_TC_STATS | _lib.SKA_PATH_TC_TOKEN_BWD |
                                   _lib.SKA_PATH_WARP_CHUNK | _lib.SKA_PATH_TC_READOUT_BWD |
                                   _lib.SKA_PATH_FUSED_SCAN | _lib.SKA_PATH_TC_READOUT_FWD |
                                   _lib.SKA_PATH_TC_CHUNK_FWD | _lib.SKA_PATH_TC_CHUNK_BWD)


@pytest.mark.parametrize("alpha", [None, 0.9])
def test_fused_statistics_scan_ragged(alpha):
    """64 series (enough for the one-CTA-per-series statistics + scan kernel), a
    ragged tail chunk, the standard and the decayed scan, forward and backward,
    against the oracle."""
    from koopman_mamba_b200 import _lib
    zt = torch.empty(4, 300, 16, 32, dtype=torch.bfloat16, device=DEV)
    vt = torch.empty(4, 300, 16, 64, dtype=torch.bfloat16, device=DEV)
    assert _path(zt, vt, 32, 64) & _lib.SKA_PATH_FUSED_SCAN
    z, zq, v, dy = _inputs(4, 300, 16, 32, 64, 21)
    kw = {} if alpha is None else dict(chunk_strategy="decay", decay_alpha=alpha)
    got = run_cuda(z, zq, v, 1.1, dy, torch.bfloat16, **kw)
    zb, zqb, vb, dyb = (bf16_round(a) for a in (z, zq, v, dy))
    ref = ska_core_fwd_bwd(zb, zqb, vb, 1.1, dyb, SkaParams(decay_alpha=alpha))
    assert_close(got[:4], ref[:4], BF16_TOL)
    assert abs(got[4] - ref[4]) <= BF16_TOL * max(1.0, abs(ref[4]))


@pytest.mark.parametrize("K", [0, 1, 3])
def test_bf16_r32_short_chunks_each_power(K):
    """bf16, r = 32 with 32-token chunks (early prefixes barely above rank), a
    partial P block (P = 48), a ragged tail, 21 chunks and each A^K branch,
    forward and backward, against the oracle: the harder conditioning that pins
    the chunk algebra's precision."""
    z, zq, v, dy = _inputs(1, 200, 3, 32, 48, 11 + K)
    got = run_cuda(z, zq, v, 1.2, dy, torch.bfloat16, chunk_size=32, power_K=K)
    zb, zqb, vb, dyb = (bf16_round(a) for a in (z, zq, v, dy))
    ref = ska_core_fwd_bwd(zb, zqb, vb, 1.2, dyb, SkaParams(chunk_size=32, power_K=K))
    assert_close(got[:4], ref[:4], BF16_TOL)
    assert abs(got[4] - ref[4]) <= BF16_TOL * max(1.0, abs(ref[4]))


@pytest.mark.parametrize("r,P,K,chunk,alpha", [
    (48, 64, 0, 64, None), (48, 64, 1, 64, None), (48, 64, 2, 32, None),   # each A^K branch
    (48, 32, 2, 64, None),          # P = 32: zero rows past P in the value operands
    (64, 48, 2, 128, None),         # r = 64 (no padding), P = 48, 128-token chunks
    (48, 64, 2, 64, 0.9),           # the decayed scan
])
def test_bf16_four_warp_backward(r, P, K, chunk, alpha):
    """bf16, 32 < r <= 64: the four-warp backward from the operators the forward
    kept (SKA_PATH_QUAD_CHUNK_BWD), a ragged tail, forward and backward against the
    oracle."""
    from koopman_mamba_b200 import _lib
    zt = torch.empty(2, 300, 3, r, dtype=torch.bfloat16, device=DEV)
    vt = torch.empty(2, 300, 3, P, dtype=torch.bfloat16, device=DEV)
    assert _path(zt, vt, r, P, chunk, power_K=K) & _lib.SKA_PATH_QUAD_CHUNK_BWD
    z, zq, v, dy = _inputs(2, 300, 3, r, P, 50 + r + K)
    kw = {} if alpha is None else dict(chunk_strategy="decay", decay_alpha=alpha)
    got = run_cuda(z, zq, v, 1.2, dy, torch.bfloat16, chunk_size=chunk, power_K=K, **kw)
    zb, zqb, vb, dyb = (bf16_round(a) for a in (z, zq, v, dy))
    ref = ska_core_fwd_bwd(zb, zqb, vb, 1.2, dyb, SkaParams(chunk_size=chunk, power_K=K, decay_alpha=alpha))
    assert_close(got[:4], ref[:4], BF16_TOL)
    assert abs(got[4] - ref[4]) <= BF16_TOL * max(1.0, abs(ref[4]))


def _fwd_raw(shape, z, zq, v, g, y, saved, nbytes):
    import ctypes
    from koopman_mamba_b200 import _lib
    from koopman_mamba_b200.ska import _tensor_desc
    return _lib.lib().ska_fwd(ctypes.byref(shape), _lib.SKA_DTYPE_BF16, ctypes.byref(_tensor_desc(z)),
                              ctypes.byref(_tensor_desc(zq)), ctypes.byref(_tensor_desc(v)),
                              ctypes.c_void_p(g.data_ptr()), ctypes.byref(_tensor_desc(y)),
                              ctypes.c_void_p(saved.data_ptr()), nbytes,
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("r,P", [(32, 64), (48, 64), (64, 64), (16, 32)])
def test_forward_only_buffer_gives_the_same_y(r, P):
    """A forward given only ska_forward_workspace_size bytes (no chunk operators
    kept) writes the same y, bitwise, as one given the whole saved buffer; fewer
    bytes than that are refused."""
    from koopman_mamba_b200 import _lib
    z, zq, v = (torch.as_tensor(a).to(DEV, torch.bfloat16) for a in _inputs(2, 500, 3, r, P, 80 + r, dy=False))
    g = torch.tensor(1.2, device=DEV)
    shape = _lib.make_shape(2, 500, 3, r, P, 64, 2, 1e-3)
    full, _ = _lib.workspace_size(shape)
    fwd = _lib.forward_workspace_size(shape)
    assert fwd < full
    ys = []
    for nbytes in (full, fwd):
        saved = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        y = torch.full((2, 500, 3, P), float("nan"), dtype=torch.bfloat16, device=DEV)
        assert _fwd_raw(shape, z, zq, v, g, y, saved, nbytes) == 0
        torch.cuda.synchronize()
        ys.append(y.float().cpu())
    assert torch.isfinite(ys[0]).all()
    assert torch.equal(ys[0], ys[1])
    saved = torch.empty(fwd - 256, dtype=torch.uint8, device=DEV)
    assert _fwd_raw(shape, z, zq, v, g, y, saved, fwd - 256) == _lib.SKA_ERR_WORKSPACE


@pytest.mark.parametrize("P", [32, 128])
def test_bf16_r32_value_widths(P):
    """r = 32 with P = 32 (operands staged in shared memory, 64-byte dY rows) and
    P = 128 (dY in two 128-byte swizzled atom columns, a 128-row dW' product),
    a ragged tail, forward and backward against the oracle."""
    z, zq, v, dy = _inputs(2, 333, 4, 32, P, 30 + P)
    got = run_cuda(z, zq, v, 1.1, dy, torch.bfloat16)
    zb, zqb, vb, dyb = (bf16_round(a) for a in (z, zq, v, dy))
    ref = ska_core_fwd_bwd(zb, zqb, vb, 1.1, dyb, SkaParams())
    assert_close(got[:4], ref[:4], BF16_TOL)
    assert abs(got[4] - ref[4]) <= BF16_TOL * max(1.0, abs(ref[4]))


def test_deterministic_bitwise():
    z, zq, v, dy = _inputs(2, 700, 3, 32, 64, 9)
    a = run_cuda(z, zq, v, 1.2, dy, torch.bfloat16)
    b = run_cuda(z, zq, v, 1.2, dy, torch.bfloat16)
    for x, y in zip(a, b):
        assert np.array_equal(np.asarray(x), np.asarray(y))


def test_causality_and_linearity_full_size():
    """Size-independent properties at config-2 size: v only feeds later chunks (so
    chunks <= c are bitwise unchanged when v changes in chunk c), chunk 0 is exactly
    zero, and y is linear in v."""
    z, zq, v, _ = _inputs(8, 2048, 12, 32, 64, 1)
    kw = dict(chunk_size=64)
    (y0,) = run_cuda(z, zq, v, 1.0, None, torch.bfloat16, **kw)
    assert np.all(y0[:, :64] == 0)
    v2 = v.copy()
    v2[:, 5 * 64:6 * 64] = bf16_round(v2[:, 5 * 64:6 * 64] * -3.0)
    (y1,) = run_cuda(z, zq, v2, 1.0, None, torch.bfloat16, **kw)
    assert np.array_equal(y0[:, :6 * 64], y1[:, :6 * 64])
    assert not np.array_equal(y0[:, 6 * 64:], y1[:, 6 * 64:])
    (y2,) = run_cuda(z, zq, 2.0 * v, 1.0, None, torch.bfloat16, **kw)   # exact in bf16
    assert rel_fro(y2, 2.0 * y0) <= 1e-2


def test_module_end_to_end_against_reference_fixture():
    d = load("module_small")
    m = SKAModule(int(d["meta_d_model"]), int(d["meta_H"]), rank=int(d["meta_r"]),
                  chunk_size=int(d["meta_CS"])).to(DEV)
    m.load_state_dict({k[3:]: torch.from_numpy(v) for k, v in d.items() if k.startswith("sd_")})
    x = torch.from_numpy(d["x"]).to(DEV).requires_grad_(True)
    out = m(x)
    out.backward(torch.from_numpy(d["dout"]).to(DEV))
    assert rel_fro(out.detach().cpu().numpy(), d["out"]) <= FP32_TOL
    assert rel_fro(x.grad.cpu().numpy(), d["dx"]) <= FP32_TOL
    for name, p in m.named_parameters():
        ref = d["grad_" + name]
        got = p.grad.detach().cpu().numpy()
        if got.ndim == 0:
            assert abs(float(got) - float(ref)) <= 2e-4 * max(1.0, abs(float(ref))), name
        else:
            assert rel_fro(got, ref) <= FP32_TOL, name


def test_empty_batch_and_errors():
    z = torch.zeros(0, 64, 2, 16, device=DEV, requires_grad=True)
    v = torch.zeros(0, 64, 2, 32, device=DEV, requires_grad=True)
    g = torch.tensor(1.0, device=DEV, requires_grad=True)
    y = ska_core(z, z, v, g)
    assert y.shape == (0, 64, 2, 32)
    y.sum().backward()
    assert float(g.grad) == 0.0
    with pytest.raises(SkaError):
        ska_core(torch.zeros(1, 8, 1, 65, device=DEV), torch.zeros(1, 8, 1, 65, device=DEV),
                 torch.zeros(1, 8, 1, 8, device=DEV), g)
    with pytest.raises(SkaError):
        ska_core(torch.zeros(1, 0, 1, 8, device=DEV), torch.zeros(1, 0, 1, 8, device=DEV),
                 torch.zeros(1, 0, 1, 8, device=DEV), g)


@pytest.mark.parametrize("B,T,H,r,P,chunk", [
    (4, 1024, 4, 16, 32, 64),     # config 5's SKA head (d_model 128, H=4, r=16), 16 series
    (2, 2048, 7, 48, 64, 64),     # config 4's SKA layer (H=7, r=48, the module default rank)
])
def test_bf16_model_config_heads(B, T, H, r, P, chunk):
    """The SKA shapes of the two full-model configurations, bf16, forward and backward
    against the oracle: r = 16 takes every tensor-core kernel but the fused
    statistics + scan; r = 48 the tensor-core statistics, readout, readout gradient
    and token backward around the four-warp chunk operators, forward and backward."""
    from koopman_mamba_b200 import _lib
    zt = torch.empty(B, T, H, r, dtype=torch.bfloat16, device=DEV)
    vt = torch.empty(B, T, H, P, dtype=torch.bfloat16, device=DEV)
    path = _path(zt, vt, r, P, chunk)
    assert path & _lib.SKA_PATH_TC_STATS and path & _lib.SKA_PATH_TC_TOKEN_BWD
    assert path & _lib.SKA_PATH_TC_READOUT_BWD
    if r > 32:
        assert path & _lib.SKA_PATH_QUAD_CHUNK_BWD
    z, zq, v, dy = _inputs(B, T, H, r, P, 70 + r)
    got = run_cuda(z, zq, v, 1.15, dy, torch.bfloat16, chunk_size=chunk)
    ref = ska_core_fwd_bwd(z, zq, v, 1.15, dy, SkaParams(chunk_size=chunk), np.float32)
    assert_close(got[:4], ref[:4], BF16_TOL)
    assert abs(got[4] - ref[4]) <= BF16_TOL * max(1.0, abs(ref[4]))


def test_module_under_bf16_autocast_against_reference_fixture():
    """SKAModule under torch.autocast(bfloat16) (fp32 hidden states, bf16 projections,
    so the core runs with bf16 I/O) against the reference module run with the same
    bf16-rounded projections (tests/golden/module_small_bf16proj.npz, fp64
    elsewhere): output, dx and every weight gradient within the bf16 bar.

    d(eta) is the dot product <d(eta y), y> of ~51K terms that cancel (on this
    fixture their magnitudes sum to thousands of times the result), so under
    autocast its value is set by where the bf16 GEMM of out_proj's backward rounds
    d(eta y): the reference's own autocast epilogue (d(eta y) = bf16(dout W_o)),
    emulated here on the CPU from the oracle's y_hat, moves it by ~5% from its fp64
    value, and any other valid rounding order lands elsewhere in that band.  It is
    checked against that emulation within three times the rounding-noise scale
    2^-9 ||d(eta y) * y||_2; the fp32 module test pins d(eta) at 1e-4."""
    d = load("module_small_bf16proj")
    m = SKAModule(int(d["meta_d_model"]), int(d["meta_H"]), rank=int(d["meta_r"]),
                  chunk_size=int(d["meta_CS"])).to(DEV)
    m.load_state_dict({k[3:]: torch.from_numpy(v) for k, v in d.items() if k.startswith("sd_")})
    x = torch.from_numpy(d["x"]).to(DEV).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = m(x)
    assert out.dtype == torch.bfloat16
    out.float().backward(torch.from_numpy(d["dout"]).to(DEV))
    assert rel_fro(out.detach().float().cpu().numpy(), d["out"]) <= BF16_TOL
    assert rel_fro(x.grad.cpu().numpy(), d["dx"]) <= BF16_TOL
    for name, p in m.named_parameters():
        got = p.grad.detach().float().cpu().numpy()
        if got.ndim == 0:
            continue
        assert rel_fro(got, d["grad_" + name]) <= BF16_TOL, name
    # ssn_gamma: the core's own scalar (fp32 reduction of the backward kernels)
    ref_g = float(d["grad_ssn_gamma"])
    assert abs(float(m.ssn_gamma.grad) - ref_g) <= BF16_TOL * max(1.0, abs(ref_g))
    # eta: against the reference's autocast epilogue, emulated from the oracle's y_hat
    B, T, dm = d["x"].shape
    H, r = int(d["meta_H"]), int(d["meta_r"])
    P = dm // H
    bf = lambda a: torch.as_tensor(a, dtype=torch.float64).bfloat16().double()   # noqa: E731
    xs = torch.as_tensor(d["x"], dtype=torch.float64)
    proj = [bf(xs @ torch.as_tensor(d["sd_" + k + ".weight"], dtype=torch.float64).T)
            for k in ("key_proj", "query_proj", "value_proj")]
    y, _ = ska_core_forward(proj[0].reshape(B, T, H, r).numpy(), proj[1].reshape(B, T, H, r).numpy(),
                            proj[2].reshape(B, T, H, P).numpy(), float(d["sd_ssn_gamma"]),
                            SkaParams(chunk_size=int(d["meta_CS"])))
    g = bf(bf(d["dout"]).numpy() @ bf(d["sd_out_proj.weight"]).numpy())       # bf16(dout W_o)
    terms = g.numpy() * y.reshape(B, T, H * P)
    deta_ref_autocast = float(terms.sum())
    noise = 2.0 ** -9 * float(np.sqrt((terms ** 2).sum()))
    assert abs(float(m.eta.grad) - deta_ref_autocast) <= 3.0 * noise, \
        (float(m.eta.grad), deta_ref_autocast, float(d["grad_eta"]), noise)


def test_module_fused_projection_matches_separate_projections():
    """The module's one-GEMM projection path gives what three separate projections
    through ska_core give (fp32, forward and every gradient)."""
    torch.manual_seed(11)
    m = SKAModule(96, 3, rank=16, chunk_size=32).to(DEV)
    with torch.no_grad():
        m.out_proj.weight.normal_(0, 0.05)
        m.ssn_gamma.fill_(1.2)
    x = torch.randn(2, 150, 96, device=DEV, requires_grad=True)
    dout = torch.randn(2, 150, 96, device=DEV)
    out = m(x)
    out.backward(dout)
    g1 = [x.grad.clone()] + [p.grad.clone() for p in m.parameters()]
    x.grad = None
    m.zero_grad()
    B, T, _ = x.shape
    z = m.key_proj(x).reshape(B, T, 3, 16)
    zq = m.query_proj(x).reshape(B, T, 3, 16)
    v = m.value_proj(x).reshape(B, T, 3, 32)
    y = ska_core(z, zq, v, m.ssn_gamma, chunk_size=32)
    out2 = m.out_proj(m.eta * y.reshape(B, T, 96))
    out2.backward(dout)
    g2 = [x.grad] + [p.grad for p in m.parameters()]
    assert rel_fro(out.detach().cpu().numpy(), out2.detach().cpu().numpy()) <= 1e-5
    for a, b in zip(g1, g2):
        assert rel_fro(a.cpu().numpy(), b.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("r,P,chunk", [(32, 64, 64), (64, 64, 128), (16, 32, 64)])
def test_bf16_inputs_fp32_y(r, P, chunk):
    """SKA_DTYPE_BF16_Y32: bf16 z, zq, v with an fp32 y (the autocast setting of the
    reference module).  Everything after the bf16 inputs is fp32-level, so y meets
    the fp32 bar against the oracle on the same bf16-rounded inputs; the bf16-y run
    agrees with it to bf16 rounding.  A layout that does not reach the tensor-core
    readout (r = 20) is refused."""
    import ctypes
    from koopman_mamba_b200 import _lib
    B, T, H = 2, 300, 3
    z, zq, v = _inputs(B, T, H, r, P, 80 + r, dy=False)
    t = [torch.as_tensor(a).to(DEV, torch.bfloat16) for a in (z, zq, v)]
    shape = _lib.make_shape(B, T, H, r, P, chunk, 2, 1e-3)
    saved_bytes, _ = _lib.workspace_size(shape)
    saved = torch.empty(saved_bytes, dtype=torch.uint8, device=DEV)
    g = torch.tensor(1.1, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    d = lambda x: _lib.SkaTensor(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2))   # noqa: E731
    outs = {}
    for code, dt in ((_lib.SKA_DTYPE_BF16_Y32, torch.float32), (_lib.SKA_DTYPE_BF16, torch.bfloat16)):
        y = torch.empty(B, T, H, P, dtype=dt, device=DEV)
        _lib.check("ska_fwd", _lib.lib().ska_fwd(ctypes.byref(shape), code, *[ctypes.byref(d(x)) for x in t],
                                                 ctypes.c_void_p(g.data_ptr()), ctypes.byref(d(y)),
                                                 ctypes.c_void_p(saved.data_ptr()), saved_bytes, stream))
        torch.cuda.synchronize()
        outs[dt] = y.double().cpu().numpy()
    ref, _ = ska_core_forward(z, zq, v, 1.1, SkaParams(chunk_size=chunk))
    assert rel_fro(outs[torch.float32], ref) <= FP32_TOL
    assert rel_fro(outs[torch.bfloat16], outs[torch.float32]) <= 4e-3
    # no tensor-core readout for r = 20: refused, nothing launched
    s20 = _lib.make_shape(B, T, H, 20, P, chunk, 2, 1e-3)
    z20 = torch.zeros(B, T, H, 20, dtype=torch.bfloat16, device=DEV)
    y = torch.empty(B, T, H, P, dtype=torch.float32, device=DEV)
    sb20, _ = _lib.workspace_size(s20)
    saved20 = torch.empty(sb20, dtype=torch.uint8, device=DEV)
    rc = _lib.lib().ska_fwd(ctypes.byref(s20), _lib.SKA_DTYPE_BF16_Y32, ctypes.byref(d(z20)), ctypes.byref(d(z20)),
                            ctypes.byref(d(t[2])), ctypes.c_void_p(g.data_ptr()), ctypes.byref(d(y)),
                            ctypes.c_void_p(saved20.data_ptr()), sb20, stream)
    assert rc == _lib.SKA_ERR_UNSUPPORTED
