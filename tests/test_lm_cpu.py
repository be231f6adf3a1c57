"""CPU: host-side checks of the hybrid Mamba-2 + SKA language model: the layer
layout and hyper-parameters of the configuration-4 model, and the Mamba-2
stand-in's chunked SSD scan against the plain sequential recurrence."""
import torch

from koopman_mamba_b200.lm import (HybridLM, Mamba2Block, SKABlock, _ssd_scan, config_50m_mamba_ska,
                                   config_mqar_2layer)


def test_config4_layout_and_parameters():
    cfg = config_50m_mamba_ska()
    m = HybridLM(cfg)
    kinds = ["S" if isinstance(layer, SKABlock) else "M" for layer in m.seq_layers]
    assert "".join(kinds) == "MMSMMSMMSMMM"            # SKA where the 50M config puts attention
    assert all(isinstance(m.seq_layers[i], Mamba2Block) for i in (0, 1, 3, 11))
    ska = m.seq_layers[2].ska
    assert (ska.H, ska.rank, ska.P, ska.chunk_size, ska.d_model) == (7, 48, 64, 64, 448)
    assert m.lm_head.weight is m.embed.weight            # tied embeddings
    n = sum(p.numel() for p in m.parameters())
    assert 40e6 < n < 60e6, n                             # the ~50M-parameter configuration


def test_mqar_2layer_layout():
    m = HybridLM(config_mqar_2layer())
    assert isinstance(m.seq_layers[0], Mamba2Block) and isinstance(m.seq_layers[1], SKABlock)
    ska = m.seq_layers[1].ska
    assert (ska.H, ska.rank, ska.P, ska.d_model) == (4, 16, 32, 128)


def test_ssd_scan_matches_the_recurrence():
    torch.manual_seed(0)
    B, L, H, P, N, Q = 2, 96, 3, 8, 5, 32
    x = torch.randn(B, L, H, P, dtype=torch.float64)
    a = -torch.rand(B, L, H, dtype=torch.float64) * 0.5
    b = torch.randn(B, L, N, dtype=torch.float64)
    c = torch.randn(B, L, N, dtype=torch.float64)
    y = _ssd_scan(x, a, b, c, Q)
    h = torch.zeros(B, H, P, N, dtype=torch.float64)
    ref = []
    for t in range(L):
        h = torch.exp(a[:, t])[..., None, None] * h + x[:, t][..., None] * b[:, t][:, None, None, :]
        ref.append(torch.einsum("bhpn,bn->bhp", h, c[:, t]))
    ref = torch.stack(ref, 1)
    assert float((y - ref).abs().max() / ref.abs().max()) < 1e-6   # decays are carried in fp32
