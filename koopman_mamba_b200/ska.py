"""Drop-in Spectral Koopman Attention module backed by the sm_100a SKA kernels.

Mirrors ``koopman_lm.ska.SKAModule`` (upstream ``koopman-lm-fast/koopman_lm/ska.py:337-476``):
the same constructor arguments, parameter names, initialisation, state-dict
keys, attributes and ``forward(hidden_states[B,T,d_model]) -> [B,T,d_model]``.
The projections (``ska.py:428-430``) and the ``eta`` / ``out_proj`` epilogue
(``ska.py:459-460``) stay PyTorch; everything between them (fp32 upcast,
shared max-key-norm scaling, chunk statistics, exclusive scan, Cholesky with
jitter, spectral normalisation, filter, readout, and the whole backward) runs in
``libska_b200.so`` through its C ABI.  There is no other implementation to
fall back to: CPU tensors raise.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn as nn

from . import _lib

__all__ = ["SKAModule", "ska_core", "SkaCoreFunction", "ProjectedSkaFunction"]

_DTYPES = {torch.float32: _lib.SKA_DTYPE_F32, torch.bfloat16: _lib.SKA_DTYPE_BF16}


def _tensor_desc(x: torch.Tensor) -> _lib.SkaTensor:
    if x.dim() != 4:
        raise ValueError(f"expected a [B,T,H,D] tensor, got shape {tuple(x.shape)}")
    if x.numel() > 0 and x.shape[-1] > 1 and x.stride(-1) != 1:
        raise ValueError("the feature (last) dimension must be contiguous")
    return _lib.SkaTensor(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2))


def _feature_contiguous(x: torch.Tensor) -> torch.Tensor:
    if x.numel() == 0 or x.shape[-1] <= 1 or x.stride(-1) == 1:
        return x
    return x.contiguous()


class _Params:
    __slots__ = ("chunk_size", "ridge_eps", "power_K", "strategy", "decay_alpha")

    def __init__(self, chunk_size, ridge_eps, power_K, strategy, decay_alpha):
        self.chunk_size = int(chunk_size)
        self.ridge_eps = float(ridge_eps)
        self.power_K = int(power_K)
        self.strategy = int(strategy)
        self.decay_alpha = float(decay_alpha)


def _shape(z, v, p: _Params) -> _lib.SkaShape:
    B, T, H, r = z.shape
    return _lib.make_shape(B, T, H, r, v.shape[-1], p.chunk_size, p.power_K, p.ridge_eps,
                           p.strategy, p.decay_alpha)


def _check_inputs(z, zq, v, gamma):
    for name, t in (("z", z), ("zq", zq), ("v", v)):
        if not t.is_cuda:
            raise RuntimeError(f"SKA core: {name} is on {t.device}; the SKA core runs only on CUDA "
                               "(sm_100a) devices")
    if not (z.device == zq.device == v.device):
        raise RuntimeError("SKA core: z, zq, v must be on the same device")
    if z.dtype not in _DTYPES:
        raise TypeError(f"SKA core: unsupported dtype {z.dtype} (float32 or bfloat16)")
    if not (z.dtype == zq.dtype == v.dtype):
        raise TypeError("SKA core: z, zq, v must share one dtype")
    if z.shape != zq.shape or z.shape[:3] != v.shape[:3]:
        raise ValueError(f"SKA core: shape mismatch z{tuple(z.shape)} zq{tuple(zq.shape)} v{tuple(v.shape)}")
    if gamma.numel() != 1:
        raise ValueError("SKA core: ssn_gamma must be a scalar")


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _y32_ok(z, v, params: _Params) -> bool:
    """bf16 z, zq, v whose layout reaches the tensor-core readout, which can write an
    fp32 y (SKA_DTYPE_BF16_Y32)."""
    if z.dtype != torch.bfloat16:
        return False
    shape = _shape(z, v, params)
    mask = _lib.lib().ska_kernel_path(ctypes.byref(shape), _lib.SKA_DTYPE_BF16, ctypes.byref(_tensor_desc(z)),
                                      ctypes.byref(_tensor_desc(v)))
    return mask >= 0 and bool(mask & _lib.SKA_PATH_TC_READOUT_FWD)


def _core_fwd(z, zq, v, g32, params: _Params, y32: bool = False, for_backward: bool = True):
    """ska_fwd on caller-owned tensors; returns (y, saved, saved_bytes, scratch_bytes).
    y32: bf16 inputs with an fp32 y (the caller checked _y32_ok).  for_backward=False:
    the smaller forward-only saved buffer (no chunk operators kept for ska_bwd)."""
    dev = z.device
    shape = _shape(z, v, params)
    saved_bytes, scratch_bytes = _lib.workspace_size(shape)
    if not for_backward:
        saved_bytes = _lib.forward_workspace_size(shape)
    B, T, H, _ = z.shape
    y = torch.empty((B, T, H, v.shape[-1]), dtype=torch.float32 if y32 else z.dtype, device=dev)
    saved = torch.empty(max(saved_bytes, 1), dtype=torch.uint8, device=dev)
    dz_, dzq_, dv_, dy_ = (_tensor_desc(t) for t in (z, zq, v, y))
    io = _lib.SKA_DTYPE_BF16_Y32 if y32 else _DTYPES[z.dtype]
    with torch.cuda.device(dev):
        rc = _lib.lib().ska_fwd(ctypes.byref(shape), io, ctypes.byref(dz_),
                                ctypes.byref(dzq_), ctypes.byref(dv_), ctypes.c_void_p(g32.data_ptr()),
                                ctypes.byref(dy_), ctypes.c_void_p(saved.data_ptr()), saved_bytes,
                                ctypes.c_void_p(_stream_ptr(dev)))
    _lib.check("ska_fwd", rc)
    return y, saved, saved_bytes, scratch_bytes


def _core_bwd(z, zq, v, g32, dy, params: _Params, saved, saved_bytes, scratch_bytes, dz, dzq, dv):
    """ska_bwd writing into the caller's dz, dzq, dv (any feature-contiguous views);
    returns d(gamma) as a float32 scalar tensor."""
    dev = z.device
    shape = _shape(z, v, params)
    scratch = torch.empty(max(scratch_bytes, 1), dtype=torch.uint8, device=dev)
    dgamma = torch.empty((), dtype=torch.float32, device=dev)
    descs = [_tensor_desc(t) for t in (z, zq, v, dy, dz, dzq, dv)]
    with torch.cuda.device(dev):
        rc = _lib.lib().ska_bwd(ctypes.byref(shape), _DTYPES[z.dtype], ctypes.byref(descs[0]),
                                ctypes.byref(descs[1]), ctypes.byref(descs[2]),
                                ctypes.c_void_p(g32.data_ptr()), ctypes.byref(descs[3]),
                                ctypes.c_void_p(saved.data_ptr()), saved_bytes,
                                ctypes.c_void_p(scratch.data_ptr()), scratch_bytes,
                                ctypes.byref(descs[4]), ctypes.byref(descs[5]), ctypes.byref(descs[6]),
                                ctypes.c_void_p(dgamma.data_ptr()), ctypes.c_void_p(_stream_ptr(dev)))
    _lib.check("ska_bwd", rc)
    return dgamma


def _gamma32(gamma, dev):
    return gamma.detach().reshape(()).to(device=dev, dtype=torch.float32).contiguous()


class SkaCoreFunction(torch.autograd.Function):
    """autograd wrapper: forward = ``ska_fwd``, backward = ``ska_bwd``."""

    @staticmethod
    def forward(ctx, z, zq, v, gamma, params: _Params):
        _check_inputs(z, zq, v, gamma)
        z, zq, v = (_feature_contiguous(t) for t in (z, zq, v))
        g32 = _gamma32(gamma, z.device)
        y, saved, ctx.saved_bytes, ctx.scratch_bytes = _core_fwd(z, zq, v, g32, params,
                                                                 for_backward=any(ctx.needs_input_grad[:4]))
        ctx.params = params
        ctx.gamma_dtype = gamma.dtype
        ctx.gamma_shape = gamma.shape
        ctx.save_for_backward(z, zq, v, g32, saved)
        return y

    @staticmethod
    def backward(ctx, dy):
        z, zq, v, g32, saved = ctx.saved_tensors
        dy = _feature_contiguous(dy.to(z.dtype))
        dz = torch.empty_like(z, memory_format=torch.contiguous_format)
        dzq = torch.empty_like(zq, memory_format=torch.contiguous_format)
        dv = torch.empty_like(v, memory_format=torch.contiguous_format)
        dgamma = _core_bwd(z, zq, v, g32, dy, ctx.params, saved, ctx.saved_bytes, ctx.scratch_bytes, dz, dzq, dv)
        dg = dgamma.to(ctx.gamma_dtype).reshape(ctx.gamma_shape)
        return dz, dzq, dv, dg, None


def _split_proj(proj, H, r, P):
    """z, zq, v as column slices of the fused projection output [B, T, H(2r + P)]
    (views: the kernels take the strides as they are)."""
    Hr = H * r
    return (proj[..., :Hr].unflatten(-1, (H, r)), proj[..., Hr:2 * Hr].unflatten(-1, (H, r)),
            proj[..., 2 * Hr:].unflatten(-1, (H, P)))


class ProjectedSkaFunction(torch.autograd.Function):
    """The key/query/value projections as ONE GEMM ``x [Wk; Wq; Wv]^T`` whose column
    slices feed the SKA core without copies, then the core (upstream
    ``ska_fast.py:361-364`` fuses the projections the same way; ``ska.py:428-457``
    is the math).  The backward has the core write dz, dzq, dv straight into one
    gradient buffer of the fused projection's shape, then forms ``dx = dproj W`` and
    ``dW = dproj^T x`` as two GEMMs (instead of three projections' six, and without
    materialising the slices' gradients separately).  Under autocast the GEMMs run
    in the autocast dtype, as ``nn.Linear`` would."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda")
    def forward(ctx, x, w, gamma, H, r, P, params: _Params):
        proj = torch.nn.functional.linear(x, w)
        if proj.dtype not in _DTYPES:
            proj = proj.float()
        z, zq, v = _split_proj(proj, H, r, P)
        _check_inputs(z, zq, v, gamma)
        g32 = _gamma32(gamma, x.device)
        # fp32 hidden states with bf16 projections (autocast): the reference keeps the
        # core's output in fp32 (ska.py:436-458), so y is written in fp32 where the
        # tensor-core readout allows it
        y32 = x.dtype == torch.float32 and proj.dtype == torch.bfloat16 and _y32_ok(z, v, params)
        y, saved, ctx.saved_bytes, ctx.scratch_bytes = _core_fwd(z, zq, v, g32, params, y32,
                                                                 for_backward=any(ctx.needs_input_grad[:3]))
        ctx.params, ctx.hrp = params, (H, r, P)
        ctx.gamma_dtype, ctx.gamma_shape = gamma.dtype, gamma.shape
        ctx.save_for_backward(x, w, proj, g32, saved)
        return y

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, dy):
        x, w, proj, g32, saved = ctx.saved_tensors
        H, r, P = ctx.hrp
        z, zq, v = _split_proj(proj, H, r, P)
        dy = _feature_contiguous(dy.to(proj.dtype))
        dproj = torch.empty_like(proj)
        dz, dzq, dv = _split_proj(dproj, H, r, P)
        dgamma = _core_bwd(z, zq, v, g32, dy, ctx.params, saved, ctx.saved_bytes, ctx.scratch_bytes, dz, dzq, dv)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.matmul(dproj, w.to(dproj.dtype) if not torch.is_autocast_enabled() else w)
        if ctx.needs_input_grad[1]:
            x2 = x.reshape(-1, x.shape[-1])
            d2 = dproj.reshape(-1, dproj.shape[-1])
            dw = torch.matmul(d2.t(), x2.to(d2.dtype) if not torch.is_autocast_enabled() else x2)
        dg = dgamma.to(ctx.gamma_dtype).reshape(ctx.gamma_shape)
        return dx, dw, dg, None, None, None, None


def ska_core(z, zq, v, gamma, *, chunk_size=64, ridge_eps=1e-3, power_K=2, chunk_strategy="standard",
             decay_alpha=0.95):
    """SKA core ``(z, zq, v, ssn_gamma) -> y_hat`` ([B,T,H,P], dtype of ``z``).

    Equivalent to upstream ``ska.py:436-457`` (upcast, max-key-norm scaling,
    chunk statistics + Cholesky, post-Cholesky chain) for
    ``chunk_strategy`` in {'standard', 'decay'}; differentiable w.r.t. z, zq, v
    and gamma.
    """
    if not torch.is_tensor(gamma):
        gamma = torch.tensor(float(gamma), device=z.device)
    if chunk_strategy == "standard":
        strategy, alpha = _lib.SKA_STRATEGY_STANDARD, 1.0
    elif chunk_strategy == "decay":
        strategy, alpha = _lib.SKA_STRATEGY_DECAY, float(decay_alpha)
    else:
        raise NotImplementedError(f"chunk_strategy={chunk_strategy!r} is not supported by the sm_100a SKA core")
    return SkaCoreFunction.apply(z, zq, v, gamma, _Params(chunk_size, ridge_eps, power_K, strategy, alpha))


class SKAModule(nn.Module):
    """Spectral Koopman Attention with chunk-causal statistics (drop-in for the
    reference ``SKAModule``).

    Args (same meaning and defaults as upstream ``ska.py:368-371``):
        d_model, n_heads, rank=48, head_dim=None (d_model // n_heads),
        ridge_eps=1e-3, scale=1.5 (initial eta), power_K=2, chunk_size=64,
        backend='auto' (resolved to 'sm100a'; 'pytorch' / 'triton' are accepted
        for compatibility, and the core always runs on the sm_100a kernels),
        chunk_strategy='standard' | 'decay' ('overlap' raises
        NotImplementedError), overlap_fraction=0.5, decay_alpha=0.95.
    """

    def __init__(self, d_model, n_heads, rank=48, head_dim=None, ridge_eps=1e-3, scale=1.5, power_K=2,
                 chunk_size=64, backend="auto", chunk_strategy="standard", overlap_fraction=0.5,
                 decay_alpha=0.95):
        super().__init__()
        if chunk_strategy not in ("standard", "decay", "overlap"):
            raise ValueError(f"unknown chunk_strategy {chunk_strategy!r}")
        if chunk_strategy == "overlap":
            raise NotImplementedError("chunk_strategy='overlap' is not supported by the sm_100a SKA core")
        self.rank = rank
        self.ridge_eps = ridge_eps
        self.power_K = power_K
        self.H = n_heads
        self.P = head_dim or (d_model // n_heads)
        self.d_model = d_model
        self.chunk_size = chunk_size
        self.chunk_strategy = chunk_strategy
        self.overlap_fraction = overlap_fraction
        self.decay_alpha = decay_alpha
        # the reference resolves 'auto' to the backend that will run (ska.py:383-386);
        # here that is always the sm_100a kernels.  An explicit 'pytorch' or 'triton'
        # is kept as given (for extra_repr and checkpoint tooling) but runs the same
        # kernels.
        self.backend = "sm100a" if backend == "auto" else backend

        # same construction and init order as the reference (ska.py:389-400), so a
        # seeded construction gives identical weights
        self.key_proj = nn.Linear(d_model, n_heads * rank, bias=False)
        self.query_proj = nn.Linear(d_model, n_heads * rank, bias=False)
        self.value_proj = nn.Linear(d_model, n_heads * self.P, bias=False)
        self.out_proj = nn.Linear(n_heads * self.P, d_model, bias=False)

        nn.init.orthogonal_(self.key_proj.weight)
        nn.init.orthogonal_(self.query_proj.weight)
        nn.init.xavier_uniform_(self.value_proj.weight)
        nn.init.zeros_(self.out_proj.weight)

        self.eta = nn.Parameter(torch.tensor(scale))
        self.ssn_gamma = nn.Parameter(torch.tensor(1.0))

    def _params(self) -> _Params:
        if self.chunk_strategy == "standard":
            strategy, alpha = _lib.SKA_STRATEGY_STANDARD, 1.0
        else:
            strategy, alpha = _lib.SKA_STRATEGY_DECAY, float(self.decay_alpha)
        return _Params(self.chunk_size, self.ridge_eps, self.power_K, strategy, alpha)

    def forward(self, hidden_states):
        """``ska.py:423-461``: projections, SKA core, eta and out_proj.  The three
        projections run as one GEMM whose column slices go to the kernels without
        copies (ProjectedSkaFunction).  Outside autocast, eta is folded into the
        out_proj weight (``out_proj(eta y) = y (eta W_o)^T``), which saves a pass
        over y; under autocast the epilogue is the reference's (``eta * y`` in the
        hidden-state dtype, then out_proj), because folding would take d(eta)
        through the bf16-rounded weight gradient instead of through y."""
        B, T, _ = hidden_states.shape
        r, H, P = self.rank, self.H, self.P
        w = torch.cat([self.key_proj.weight, self.query_proj.weight, self.value_proj.weight], 0)
        y_hat = ProjectedSkaFunction.apply(hidden_states, w, self.ssn_gamma, H, r, P, self._params())
        y_hat = y_hat.reshape(B, T, H * P).to(hidden_states.dtype)
        if torch.is_autocast_enabled(hidden_states.device.type):
            return self.out_proj(self.eta * y_hat)
        return torch.nn.functional.linear(y_hat, self.out_proj.weight * self.eta)

    def extra_repr(self):
        parts = [
            f"d_model={self.d_model}",
            f"n_heads={self.H}",
            f"rank={self.rank}",
            f"chunk_size={self.chunk_size}",
            f"backend={self.backend}",
            f"chunk_strategy={self.chunk_strategy}",
        ]
        if self.chunk_strategy == "decay":
            parts.append(f"decay_alpha={self.decay_alpha}")
        return ", ".join(parts)
