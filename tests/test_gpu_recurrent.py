"""GPU parity of the recurrent (decode) path: ska_prefill_state and ska_step
through the C ABI against the reference's own _ska_prefill / _ska_step outputs
(tests/golden/recur_*.npz) and against the recurrent oracle.

Tolerances (relative Frobenius norm): fp32 I/O 1e-4 on the state and on every
decode output; bf16 I/O 2e-2 against the oracle fed the same bf16-rounded inputs.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from koopman_mamba_b200 import SKAModule, _lib
from koopman_mamba_b200.recurrent import SKAState, ska_prefill, ska_step
from oracle.ska_oracle import rel_fro
from oracle.ska_recurrent import decode_step, prefill_state
from tests._golden import load

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
FP32_TOL = 1e-4
BF16_TOL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _desc(t):
    return _lib.SkaTensor(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


class _Layer:
    """A layer's prefill + steps through the C ABI with caller-owned buffers."""

    def __init__(self, B, H, r, P, CS, K, ridge, gamma, dtype):
        self.B, self.H, self.r, self.P, self.CS, self.K, self.ridge = B, H, r, P, CS, K, ridge
        self.dtype = dtype
        self.io = _lib.SKA_DTYPE_F32 if dtype == torch.float32 else _lib.SKA_DTYPE_BF16
        self.gamma = torch.tensor(float(gamma), device=DEV)
        self.state = SKAState(B, H, r, P, DEV, ridge_eps=ridge)

    def shape(self, T):
        return _lib.make_shape(self.B, T, self.H, self.r, self.P, self.CS, self.K, self.ridge)

    def prefill(self, z, zq, v):
        z, zq, v = (torch.as_tensor(np.ascontiguousarray(a)).to(DEV, self.dtype) for a in (z, zq, v))
        s = self.shape(z.shape[1])
        saved_bytes, _ = _lib.workspace_size(s)
        saved = torch.empty(saved_bytes, dtype=torch.uint8, device=DEV)
        y = torch.empty(*z.shape[:3], self.P, dtype=self.dtype, device=DEV)
        L = _lib.lib()
        dz, dzq, dv, dy = (_desc(t) for t in (z, zq, v, y))
        _lib.check("ska_fwd", L.ska_fwd(ctypes.byref(s), self.io, ctypes.byref(dz), ctypes.byref(dzq),
                                        ctypes.byref(dv), ctypes.c_void_p(self.gamma.data_ptr()), ctypes.byref(dy),
                                        ctypes.c_void_p(saved.data_ptr()), saved_bytes, _stream()))
        _lib.check("ska_prefill_state", L.ska_prefill_state(
            ctypes.byref(s), self.io, ctypes.byref(dz), ctypes.byref(dv), ctypes.c_void_p(saved.data_ptr()),
            saved_bytes, ctypes.c_void_p(self.state.buffer.data_ptr()), self.state._bytes, _stream()))
        self.state._has_last = True
        return y

    def step(self, z, zq, v):
        """z, zq [B, T, H, r], v [B, T, H, P] numpy -> y [B, T, H, P] float64."""
        z, zq, v = (torch.as_tensor(np.ascontiguousarray(a)).to(DEV, self.dtype) for a in (z, zq, v))
        s = self.shape(z.shape[1])
        y = torch.empty(*z.shape[:3], self.P, dtype=self.dtype, device=DEV)
        dz, dzq, dv, dy = (_desc(t) for t in (z, zq, v, y))
        _lib.check("ska_step", _lib.lib().ska_step(
            ctypes.byref(s), self.io, ctypes.byref(dz), ctypes.byref(dzq), ctypes.byref(dv),
            ctypes.c_void_p(self.gamma.data_ptr()), ctypes.byref(dy), ctypes.c_void_p(self.state.buffer.data_ptr()),
            self.state._bytes, _stream()))
        torch.cuda.synchronize()
        return y.double().cpu().numpy()

    def host_state(self):
        torch.cuda.synchronize()
        st = self.state
        return dict(G=st.G.double().cpu().numpy(), M=st.M.double().cpu().numpy(), C=st.C_v.double().cpu().numpy(),
                    zlast=st.z_last.double().cpu().numpy(), maxnorm=st.max_norm.reshape(self.B, self.H).double().cpu().numpy())


@pytest.mark.parametrize("case", ["recur_r16", "recur_r32"])
def test_prefill_and_decode_against_reference_golden(case):
    d = load(case)
    m = {k[5:]: d[k] for k in d if k.startswith("meta_")}
    B, H, r, P = (int(m[k]) for k in ("B", "H", "r", "P"))
    layer = _Layer(B, H, r, P, int(m["CS"]), int(m["K"]), float(m["ridge"]), float(m["gamma"]), torch.float32)
    layer.prefill(d["z"], d["zq"], d["v"])
    st = layer.host_state()
    for ours, ref in (("G", "G0"), ("M", "M0"), ("C", "C0"), ("zlast", "zlast0"), ("maxnorm", "maxnorm0")):
        assert rel_fro(st[ours], d[ref]) <= FP32_TOL, ref
    for s in range(int(m["steps"])):
        y = layer.step(d["z_steps"][s][:, None], d["zq_steps"][s][:, None], d["v_steps"][s][:, None])
        assert rel_fro(y[:, 0], d["y_steps"][s]) <= FP32_TOL, s
    st = layer.host_state()
    for ours, ref in (("G", "G1"), ("M", "M1"), ("C", "C1"), ("zlast", "zlast1")):
        assert rel_fro(st[ours], d[ref]) <= FP32_TOL, ref


def _inputs(B, T, H, r, P, seed):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(64)
    return [(torch.randn(B, T, H, n, generator=g) * s).bfloat16().float().numpy() for n in (r, r, P)]


def test_several_tokens_per_call_equal_single_steps():
    """ska_step over T tokens in one call gives the bits of T calls of one token."""
    z, zq, v = _inputs(2, 130, 3, 32, 64, 41)
    zs, zqs, vs = _inputs(2, 4, 3, 32, 64, 42)
    a = _Layer(2, 3, 32, 64, 64, 2, 1e-3, 1.1, torch.float32)
    b = _Layer(2, 3, 32, 64, 64, 2, 1e-3, 1.1, torch.float32)
    a.prefill(z, zq, v)
    b.prefill(z, zq, v)
    ya = a.step(zs, zqs, vs)
    yb = np.concatenate([b.step(zs[:, t:t + 1], zqs[:, t:t + 1], vs[:, t:t + 1]) for t in range(4)], axis=1)
    assert np.array_equal(ya, yb)
    sa, sb = a.host_state(), b.host_state()
    for k in sa:
        assert np.array_equal(sa[k], sb[k]), k


@pytest.mark.parametrize("r,P,CS,T", [(32, 64, 64, 300), (16, 32, 64, 1000), (24, 48, 32, 77)])
def test_bf16_decode_against_oracle(r, P, CS, T):
    """bf16 tensors (the tensor-core prefill path at r = 32), several prompt
    lengths and head shapes, 5 decode steps against the oracle."""
    B, H = 2, 4
    z, zq, v = _inputs(B, T, H, r, P, 50 + r)
    zs, zqs, vs = _inputs(B, 5, H, r, P, 60 + r)
    layer = _Layer(B, H, r, P, CS, 2, 1e-3, 1.2, torch.bfloat16)
    layer.prefill(z, zq, v)
    ref = prefill_state(z, v, 1e-3)
    st = layer.host_state()
    for ours, theirs in (("G", ref.G), ("M", ref.M), ("C", ref.C), ("zlast", ref.z_last)):
        assert rel_fro(st[ours], theirs) <= 1e-4, ours     # bf16 tokens are exact; fp32 sums
    for s in range(5):
        y = layer.step(zs[:, s:s + 1], zqs[:, s:s + 1], vs[:, s:s + 1])
        yr = decode_step(ref, zs[:, s], zqs[:, s], vs[:, s], 1.2, 2)
        assert rel_fro(y[:, 0], yr) <= BF16_TOL, s


def test_module_prefill_and_step_against_oracle():
    """SKAModule-level prefill (layer output + state) and decode steps: the output of
    the prefill equals the module's forward, and each step equals out_proj(eta *
    the oracle's y_hat) computed from the same projections."""
    torch.manual_seed(7)
    ska = SKAModule(128, 4, rank=16, chunk_size=32).to(DEV)
    with torch.no_grad():
        ska.out_proj.weight.normal_(0, 0.05)
        ska.ssn_gamma.fill_(1.3)
    x = torch.randn(2, 90, 128, device=DEV) / 4
    out, state = ska_prefill(ska, x)
    with torch.no_grad():
        full = ska(x)
    assert rel_fro(out.double().cpu().numpy(), full.double().cpu().numpy()) <= FP32_TOL
    with torch.no_grad():
        proj = [p(x).reshape(2, 90, 4, -1).double().cpu().numpy() for p in (ska.key_proj, ska.query_proj,
                                                                             ska.value_proj)]
    ref = prefill_state(proj[0], proj[2], ska.ridge_eps)
    for _ in range(3):
        xt = torch.randn(2, 1, 128, device=DEV) / 4
        got = ska_step(ska, xt, state)
        with torch.no_grad():
            zt, zqt, vt = (p(xt).reshape(2, 4, -1).double().cpu().numpy() for p in (ska.key_proj, ska.query_proj,
                                                                                   ska.value_proj))
            yr = decode_step(ref, zt, zqt, vt, 1.3, ska.power_K)
            want = ska.out_proj(float(ska.eta) * torch.as_tensor(yr, dtype=torch.float32, device=DEV).reshape(2, 1, -1))
        assert rel_fro(got.double().cpu().numpy(), want.double().cpu().numpy()) <= FP32_TOL
    assert state.token_count == 93 and state.z_last is not None
