"""Hybrid Mamba-2 + SKA language model around the sm_100a SKA layer (full-model
integration of the drop-in SKAModule, data-parallel training with DDP).

Mirrors the reference's model assembly for the Mamba-2 + SKA variants
(upstream ``koopman-lm-fast``):

* ``koopman_lm/baselines.py:120-214`` ``_build_model`` / ``build_mamba_ska_swiglu``:
  embedding, ``n_layers`` pairs of (sequence block, SwiGLU MLP), final LayerNorm,
  LM head tied to the embedding, cross-entropy loss;
* ``koopman_lm/model.py:8-49`` ``Mamba2Block`` / ``SKABlock``: pre-LayerNorm blocks
  with a residual, the SKA block holding ``SKAModule`` with the configuration's
  SKA arguments;
* ``koopman_lm/config.py:5-64`` ``KoopmanLMConfig`` (the fields these builders
  read) and ``config_50m_mamba_attn.py:26-50`` (the configuration whose attention
  layers become SKA layers).

The SKA layers are this package's ``SKAModule`` (sm_100a kernels, gradients to
every SKA parameter).  The Mamba-2 layers use ``mamba_ssm.Mamba2`` when that
package is importable; it is not installed here, so by default they are
:class:`Mamba2Mixer`, a PyTorch layer with Mamba-2's published structure (input
projection to z, x, B, C, dt; causal depthwise convolution; the state-space
duality (SSD) scan computed chunk-wise; D skip; gated RMSNorm; output projection).
That stand-in is outside the SKA hot path: it gives the model its shape and cost,
not a reference to match.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ska import SKAModule

__all__ = ["LMConfig", "config_50m_mamba_ska", "config_mqar_2layer", "HybridLM", "Mamba2Mixer", "SwiGLUMLP"]


@dataclass
class LMConfig:
    """The fields of the reference's ``KoopmanLMConfig`` that the Mamba-2 + SKA
    builders read (same names and defaults, ``koopman_lm/config.py:5-42``)."""

    d_model: int = 768
    n_layers: int = 24
    vocab_size: int = 32000
    d_state: int = 128
    d_conv: int = 4
    mamba_expand: int = 2
    mamba_headdim: int = 64
    ska_n_heads: int = 12
    ska_rank: int = 48
    ska_ridge: float = 1e-3
    ska_scale: float = 1.5
    ska_power_K: int = 2
    ska_chunk_size: int = 64
    ska_backend: str = "auto"
    ska_chunk_strategy: str = "standard"
    ska_overlap_fraction: float = 0.5
    ska_decay_alpha: float = 0.95
    mlp_expand: float = 2.667
    ska_layer_indices: List[int] = field(default_factory=lambda: [4, 8, 12, 16, 20, 23])
    max_seq_len: int = 8192
    tie_embeddings: bool = True

    @property
    def head_dim(self):
        return self.d_model // self.ska_n_heads


def config_50m_mamba_ska() -> LMConfig:
    """``config_50m_mamba_attn.py:26-50`` with its attention layers (indices 2, 5,
    8) as SKA layers: d_model 448, 12 layers, 7 SKA heads of 64, rank 48,
    d_state 128, vocab 32000, sequences of 2048, tied embeddings."""
    return LMConfig(d_model=448, n_layers=12, vocab_size=32000, d_state=128, d_conv=4, mamba_expand=2,
                    ska_n_heads=7, ska_rank=48, ska_layer_indices=[2, 5, 8], mlp_expand=2.667,
                    max_seq_len=2048, tie_embeddings=True)


def config_mqar_2layer(vocab_size: int = 8192) -> LMConfig:
    """A 2-layer Mamba-2 + SKA model (d_model 128, SKA H=4, r=16): layer 0 Mamba-2
    (the first layer always is, ``model.py:63``), layer 1 SKA."""
    return LMConfig(d_model=128, n_layers=2, vocab_size=vocab_size, d_state=64, ska_n_heads=4, ska_rank=16,
                    ska_layer_indices=[1], max_seq_len=1024)


class _GatedRMSNorm(nn.Module):
    """rms_norm(y * silu(z)) * weight, the output norm of a Mamba-2 layer."""

    def __init__(self, d, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, y, z):
        y = y * F.silu(z)
        y = y.float()
        y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(z.dtype)


def _ssd_scan(x, a, b, c, chunk):
    """The SSD recurrence  h_t = exp(a_t) h_{t-1} + b_t x_t^T,  y_t = h_t^T c_t
    (per head; b, c shared over heads), computed chunk-wise: within a chunk as a
    masked (decay-weighted) attention-like product, across chunks by carrying the
    chunk-end states.  x [B,L,H,P] (already scaled by dt), a [B,L,H] (= A dt <= 0),
    b, c [B,L,N]; L a multiple of `chunk`.  Returns y [B,L,H,P]."""
    Bsz, L, H, P = x.shape
    N = b.shape[-1]
    nc = L // chunk
    x = x.reshape(Bsz, nc, chunk, H, P)
    a = a.reshape(Bsz, nc, chunk, H).permute(0, 3, 1, 2).float()          # [B,H,c,Q]
    b = b.reshape(Bsz, nc, chunk, N)
    c = c.reshape(Bsz, nc, chunk, N)
    acs = torch.cumsum(a, dim=-1)                                           # within-chunk log decay
    # decay from position s to position t inside a chunk (t >= s): exp(acs_t - acs_s)
    diff = acs[..., :, None] - acs[..., None, :]
    causal = torch.ones(chunk, chunk, dtype=torch.bool, device=x.device).tril()
    decay = torch.exp(diff.masked_fill(~causal, float("-inf"))).to(x.dtype)   # [B,H,c,Q,Q]
    scores = torch.matmul(c, b.transpose(-1, -2))                          # [B,c,Q,Q]
    xh = x.permute(0, 3, 1, 2, 4)                                          # [B,H,c,Q,P]
    y_in = torch.matmul(scores[:, None] * decay, xh)                       # [B,H,c,Q,P]
    # state at the end of each chunk from that chunk alone: sum_s exp(acs_end - acs_s) b_s x_s^T
    w_end = torch.exp(acs[..., -1:] - acs).to(x.dtype)                     # [B,H,c,Q]
    st_local = torch.matmul((xh * w_end[..., None]).transpose(-1, -2), b[:, None])   # [B,H,c,P,N]
    # carry across chunks: S_c = exp(chunk decay) S_{c-1} + local_c (state entering chunk c is S_{c-1})
    chunk_decay = torch.exp(acs[..., -1])                                  # [B,H,c]
    carried = []
    s = torch.zeros(Bsz, H, P, N, dtype=torch.float32, device=x.device)
    for ci in range(nc):
        carried.append(s)
        s = chunk_decay[..., ci, None, None] * s + st_local[:, :, ci].float()
    s_in = torch.stack(carried, dim=2).to(x.dtype)                         # [B,H,c,P,N]
    # contribution of the carried state: exp(acs_t) c_t^T S_in
    y_out = torch.matmul(c[:, None], s_in.transpose(-1, -2)) * torch.exp(acs)[..., None].to(x.dtype)
    y = (y_in + y_out).permute(0, 2, 3, 1, 4).reshape(Bsz, L, H, P)
    return y


class Mamba2Mixer(nn.Module):
    """A Mamba-2 layer in PyTorch (stand-in for ``mamba_ssm.Mamba2`` with one B/C
    group): in_proj -> (z, x, B, C, dt); causal depthwise conv + SiLU on (x, B, C);
    dt = softplus(dt + dt_bias), A = -exp(A_log); the SSD scan; D skip; gated
    RMSNorm; out_proj."""

    def __init__(self, d_model, d_state=128, d_conv=4, expand=2, headdim=64, chunk=64):
        super().__init__()
        self.d_inner = expand * d_model
        self.d_state = d_state
        self.headdim = headdim
        self.nheads = self.d_inner // headdim
        self.chunk = chunk
        conv_dim = self.d_inner + 2 * d_state
        self.in_proj = nn.Linear(d_model, 2 * self.d_inner + 2 * d_state + self.nheads, bias=False)
        self.conv1d = nn.Conv1d(conv_dim, conv_dim, d_conv, groups=conv_dim, padding=d_conv - 1, bias=True)
        dt = torch.exp(torch.rand(self.nheads) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))         # softplus^-1(dt)
        self.A_log = nn.Parameter(torch.log(torch.empty(self.nheads).uniform_(1, 16)))
        self.D = nn.Parameter(torch.ones(self.nheads))
        self.norm = _GatedRMSNorm(self.d_inner)
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=False)

    def forward(self, u):
        Bsz, L, _ = u.shape
        zxbcdt = self.in_proj(u)
        z, xbc, dt = torch.split(zxbcdt, [self.d_inner, self.d_inner + 2 * self.d_state, self.nheads], dim=-1)
        xbc = F.silu(self.conv1d(xbc.transpose(1, 2))[..., :L].transpose(1, 2))
        x, b, c = torch.split(xbc, [self.d_inner, self.d_state, self.d_state], dim=-1)
        dt = F.softplus(dt.float() + self.dt_bias)                            # [B,L,H]
        A = -torch.exp(self.A_log.float())
        x = x.reshape(Bsz, L, self.nheads, self.headdim)
        pad = (-L) % self.chunk
        xs, a, bs, cs = x * dt[..., None].to(x.dtype), A * dt, b, c
        if pad:
            xs, a, bs, cs = (F.pad(t, (0, 0) * (t.dim() - 2) + (0, pad)) for t in (xs, a, bs, cs))
        y = _ssd_scan(xs, a, bs, cs, self.chunk)[:, :L]
        y = y + x * self.D[:, None].to(x.dtype)
        return self.out_proj(self.norm(y.reshape(Bsz, L, self.d_inner), z))


def _mamba_layer(cfg: LMConfig):
    try:
        from mamba_ssm import Mamba2   # the reference's layer, where it is installed
        return Mamba2(d_model=cfg.d_model, d_state=cfg.d_state, d_conv=cfg.d_conv, expand=cfg.mamba_expand)
    except ImportError:
        return Mamba2Mixer(cfg.d_model, cfg.d_state, cfg.d_conv, cfg.mamba_expand, cfg.mamba_headdim)


class Mamba2Block(nn.Module):
    """``model.py:8-25``: x + mamba(LayerNorm(x))."""

    def __init__(self, cfg: LMConfig):
        super().__init__()
        self.norm = nn.LayerNorm(cfg.d_model)
        self.mamba = _mamba_layer(cfg)

    def forward(self, x):
        return x + self.mamba(self.norm(x))


class SKABlock(nn.Module):
    """``model.py:28-49``: x + ska(LayerNorm(x)) with the configuration's SKA arguments."""

    def __init__(self, cfg: LMConfig):
        super().__init__()
        self.norm = nn.LayerNorm(cfg.d_model)
        self.ska = SKAModule(d_model=cfg.d_model, n_heads=cfg.ska_n_heads, rank=cfg.ska_rank, head_dim=cfg.head_dim,
                             ridge_eps=cfg.ska_ridge, scale=cfg.ska_scale, power_K=cfg.ska_power_K,
                             chunk_size=cfg.ska_chunk_size, backend=cfg.ska_backend,
                             chunk_strategy=cfg.ska_chunk_strategy, overlap_fraction=cfg.ska_overlap_fraction,
                             decay_alpha=cfg.ska_decay_alpha)

    def forward(self, x):
        return x + self.ska(self.norm(x))


class SwiGLUMLP(nn.Module):
    """``baselines.py:27-38``: x + w3(silu(w1 h) * w2 h), h = LayerNorm(x), d_ff
    rounded up to a multiple of 64."""

    def __init__(self, d, expand=2.667):
        super().__init__()
        d_ff = ((int(d * expand) + 63) // 64) * 64
        self.norm = nn.LayerNorm(d)
        self.w1 = nn.Linear(d, d_ff, bias=False)
        self.w2 = nn.Linear(d, d_ff, bias=False)
        self.w3 = nn.Linear(d_ff, d, bias=False)

    def forward(self, x):
        h = self.norm(x)
        return x + self.w3(F.silu(self.w1(h)) * self.w2(h))


class HybridLM(nn.Module):
    """``baselines.py:120-153`` with Mamba-2 blocks and SKA blocks at
    ``cfg.ska_layer_indices``, SwiGLU MLPs, tied LM head."""

    def __init__(self, cfg: LMConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        ska_set = set(cfg.ska_layer_indices)
        self.seq_layers = nn.ModuleList(SKABlock(cfg) if i in ska_set else Mamba2Block(cfg)
                                        for i in range(cfg.n_layers))
        self.mlp_layers = nn.ModuleList(SwiGLUMLP(cfg.d_model, cfg.mlp_expand) for _ in range(cfg.n_layers))
        self.norm_f = nn.LayerNorm(cfg.d_model)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        if cfg.tie_embeddings:
            self.lm_head.weight = self.embed.weight

    def forward(self, input_ids, labels=None):
        h = self.embed(input_ids)
        for seq, mlp in zip(self.seq_layers, self.mlp_layers):
            h = mlp(seq(h))
        logits = self.lm_head(self.norm_f(h))
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), labels.reshape(-1), ignore_index=-100)
        return {"loss": loss, "logits": logits}

    def ska_parameters(self):
        """The parameters of the SKA layers (for checks that their gradients flow)."""
        return [p for layer in self.seq_layers if isinstance(layer, SKABlock) for p in layer.parameters()]
