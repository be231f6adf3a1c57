"""CPU: host-side behaviour of the drop-in SKAModule (construction, parameters,
state-dict keys, initialisation, loud failure without CUDA)."""
import numpy as np
import pytest
import torch

from koopman_mamba_b200 import SKAModule, ska_core
from tests._golden import load


def test_state_dict_keys_and_shapes_match_reference_fixture():
    d = load("module_small")
    m = SKAModule(int(d["meta_d_model"]), int(d["meta_H"]), rank=int(d["meta_r"]),
                  chunk_size=int(d["meta_CS"]))
    ref = {k[3:]: v for k, v in d.items() if k.startswith("sd_")}
    ours = m.state_dict()
    assert set(ours) == set(ref)
    for k, v in ours.items():
        assert tuple(v.shape) == tuple(ref[k].shape), k
    # loading the reference checkpoint works unchanged
    m.load_state_dict({k: torch.from_numpy(v) for k, v in ref.items()})


def test_constructor_defaults_and_attributes():
    m = SKAModule(768, 12)
    assert (m.rank, m.H, m.P, m.d_model, m.chunk_size, m.power_K) == (48, 12, 64, 768, 64, 2)
    assert m.ridge_eps == 1e-3 and m.chunk_strategy == "standard" and m.decay_alpha == 0.95
    assert float(m.eta) == 1.5 and float(m.ssn_gamma) == 1.0
    assert torch.count_nonzero(m.out_proj.weight) == 0
    w = m.key_proj.weight
    assert torch.allclose(w @ w.T, torch.eye(w.shape[0]), atol=1e-5)   # orthogonal rows
    assert "chunk_strategy=standard" in m.extra_repr()


def test_seeded_init_matches_reference_order():
    """Same construction order as upstream ska.py:389-400: equal seeds, equal weights."""
    torch.manual_seed(3)
    a = SKAModule(128, 2, rank=16)
    torch.manual_seed(3)
    lk = torch.nn.Linear(128, 32, bias=False)
    lq = torch.nn.Linear(128, 32, bias=False)
    lv = torch.nn.Linear(128, 128, bias=False)
    lo = torch.nn.Linear(128, 128, bias=False)
    torch.nn.init.orthogonal_(lk.weight)
    torch.nn.init.orthogonal_(lq.weight)
    torch.nn.init.xavier_uniform_(lv.weight)
    assert torch.equal(a.key_proj.weight, lk.weight)
    assert torch.equal(a.query_proj.weight, lq.weight)
    assert torch.equal(a.value_proj.weight, lv.weight)


def test_overlap_strategy_is_rejected_loudly():
    with pytest.raises(NotImplementedError):
        SKAModule(128, 2, rank=16, chunk_strategy="overlap")
    with pytest.raises(ValueError):
        SKAModule(128, 2, rank=16, chunk_strategy="bogus")


def test_cpu_tensors_raise_no_fallback():
    m = SKAModule(128, 2, rank=16)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 16, 128))
    z = torch.randn(1, 16, 2, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ska_core(z, z, torch.randn(1, 16, 2, 64), torch.tensor(1.0))


def test_backend_auto_resolves_like_the_reference():
    """The reference resolves backend='auto' to the backend that runs (ska.py:383-386);
    here that is always the sm_100a kernels, and explicit values are kept."""
    assert SKAModule(64, 2, rank=16).backend == "sm100a"
    assert "backend=sm100a" in SKAModule(64, 2, rank=16).extra_repr()
    assert SKAModule(64, 2, rank=16, backend="pytorch").backend == "pytorch"
