"""GPU: the SKA layer inside the hybrid Mamba-2 + SKA language model, trained with
DDP.

The reference trains this model with DistributedDataParallel and
find_unused_parameters=False (train_fast.py:255-258), but its default Triton SKA
path returns no gradient to the SKA projections, gamma or z/zq/v.  These tests
check that, with the sm_100a SKA layer, every SKA parameter receives a gradient
through a full model, that training on a fixed batch lowers the loss, and that
under DDP (two ranks, gloo, both on this GPU) the all-reduced gradients of every
parameter, SKA's included, are the average of the two ranks' single-process
gradients.
"""
import os
import tempfile

import pytest
import torch

from koopman_mamba_b200.lm import HybridLM, config_mqar_2layer

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _small_cfg():
    cfg = config_mqar_2layer(vocab_size=512)
    cfg.ska_layer_indices = [1]
    return cfg


def _batch(seed, B=4, T=256, vocab=512):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (B, T + 1), generator=g)
    return ids[:, :-1].contiguous(), ids[:, 1:].contiguous()


def _step(model, opt, ids, labels):
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = model(ids.to(DEV), labels.to(DEV))["loss"]
    opt.zero_grad(set_to_none=True)
    loss.backward()
    opt.step()
    return float(loss)


def test_every_ska_parameter_gets_a_gradient():
    torch.manual_seed(0)
    model = HybridLM(_small_cfg()).to(DEV)
    with torch.no_grad():   # gamma inside the clamp [1, 1.5] (weight decay would take 1.0 just below it,
        for layer in model.seq_layers:   # where the clamp passes no gradient, as in the reference)
            if hasattr(layer, "ska"):
                layer.ska.ssn_gamma.fill_(1.2)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    ids, labels = _batch(1)
    _step(model, opt, ids, labels)          # out_proj starts at zero (ska.py:398): one step moves it
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = model(ids.to(DEV), labels.to(DEV))["loss"]
    opt.zero_grad(set_to_none=True)
    loss.backward()
    for name, p in model.named_parameters():
        if ".ska." in name:
            assert p.grad is not None, name
            assert torch.isfinite(p.grad).all(), name
            assert float(p.grad.abs().max()) > 0, name


def test_training_lowers_the_loss():
    torch.manual_seed(1)
    model = HybridLM(_small_cfg()).to(DEV)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    ids, labels = _batch(2)
    losses = [_step(model, opt, ids, labels) for _ in range(25)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < 0.8 * losses[0], losses


def _rank_main(rank, world, path, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    torch.cuda.set_device(0)
    torch.manual_seed(0)
    model = HybridLM(_small_cfg()).to(DEV)
    with torch.no_grad():   # a non-zero out_proj, so that gradients reach the SKA core at once
        for layer in model.seq_layers:
            if hasattr(layer, "ska"):
                layer.ska.out_proj.weight.normal_(0, 0.02)
    ddp = torch.nn.parallel.DistributedDataParallel(model, device_ids=[0], find_unused_parameters=False)
    ids, labels = _batch(10 + rank)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = ddp(ids.to(DEV), labels.to(DEV))["loss"]
    loss.backward()
    torch.save({n: p.grad.detach().cpu() for n, p in model.named_parameters()}, f"{path}/rank{rank}.pt")
    dist.barrier()
    dist.destroy_process_group()


def test_ddp_all_reduces_ska_gradients():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_rank_main, args=(2, tmp, 29611), nprocs=2, start_method="spawn", join=True)
        g0 = torch.load(f"{tmp}/rank0.pt")
        g1 = torch.load(f"{tmp}/rank1.pt")
    # the same model and batches in this process, without DDP
    torch.manual_seed(0)
    model = HybridLM(_small_cfg()).to(DEV)
    with torch.no_grad():
        for layer in model.seq_layers:
            if hasattr(layer, "ska"):
                layer.ska.out_proj.weight.normal_(0, 0.02)
    per_rank = []
    for rank in range(2):
        model.zero_grad(set_to_none=True)
        ids, labels = _batch(10 + rank)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(ids.to(DEV), labels.to(DEV))["loss"]
        loss.backward()
        per_rank.append({n: p.grad.detach().cpu() for n, p in model.named_parameters()})
    n_ska = 0
    for name in g0:
        assert torch.equal(g0[name], g1[name]), name                 # all-reduced: identical on both ranks
        want = 0.5 * (per_rank[0][name] + per_rank[1][name])
        err = float((g0[name] - want).norm() / want.norm().clamp_min(1e-30))
        assert err <= 2e-2, (name, err)
        if ".ska." in name:
            n_ska += 1
            assert float(g0[name].abs().max()) > 0, name
    assert n_ska == 6   # key, query, value, out_proj weights, eta, ssn_gamma
