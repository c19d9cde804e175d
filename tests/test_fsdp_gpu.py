"""ZeRO-2 on 2 GPUs (NCCL reduce-scatter / all-gather, sharded fused optimizer with the AdamH
matrix sums all-reduced between its passes) against replicated data parallelism."""

import pytest
import torch

from mp_util import run_ranks

pytestmark = pytest.mark.gpu

CFG = dict(vocab_size=4096, hidden_dim=256, intermediate_dim=256, shared_expert_intermediate_dim=512, num_experts=8,
           num_experts_per_token=2, num_layers=2, num_heads=4, num_kv_heads=4, head_dim=64, max_seq_len=256,
           sliding_window=256, capacity_factor=4.0)


def _rank(rank, world, zero, opt="adamh"):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.optim.configs import MuonConfig
    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.parallel.fsdp import init_zero
    from marin_experiments_b200.train.trainer import Trainer

    torch.cuda.set_device(rank)
    ctx = init_zero(120) if zero else pdist.init(ep_size=1, timeout_s=120)
    try:
        o = GrugMoeAdamHConfig(warmup=0.0) if opt == "adamh" else MuonConfig(warmup=0.0, weight_decay=0.1)
        run = GrugRunConfig(model=GrugModelConfig(**CFG), optimizer=o,
                            trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=0)))
        tr = Trainer(run, device=f"cuda:{rank}", dist=ctx)
        init = tr.store.master.clone()
        tok = torch.randint(0, 4096, (2, 256), generator=torch.Generator().manual_seed(rank)).pin_memory()
        tr.train_step({"tokens": tok})
        torch.cuda.synchronize()
        return {"upd": (tr.store.master - init).cpu().numpy(), "m_numel": tr.opt.m.numel(), "n": tr.store.numel}
    finally:
        pdist.shutdown()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero_matches_dp_on_gpu():
    a = run_ranks(_rank, 2, True, timeout=300)
    b = run_ranks(_rank, 2, False, timeout=300)
    assert a[0]["m_numel"] * 2 == a[0]["n"]
    for r in range(2):
        ua, ub = torch.from_numpy(a[r]["upd"]), torch.from_numpy(b[r]["upd"])
        err = ((ua - ub).norm() / ub.norm()).item()
        assert err < 0.05, (r, err)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero_muon_matches_dp_on_gpu():
    """Muon under ZeRO on GPUs: matrices orthogonalised whole by their owner rank, crossing
    matrices handed over around the peer-memory reduce-scatter and all-gather."""
    a = run_ranks(_rank, 2, True, "muon", timeout=300)
    b = run_ranks(_rank, 2, False, "muon", timeout=300)
    for r in range(2):
        n = min(a[r]["upd"].size, b[r]["upd"].size)
        ua, ub = torch.from_numpy(a[r]["upd"][:n]), torch.from_numpy(b[r]["upd"][:n])
        err = ((ua - ub).norm() / ub.norm()).item()
        assert err < 0.05, (r, err)


def _ep_rank(rank, world, zero):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.parallel.fsdp import init_zero
    from marin_experiments_b200.train.trainer import Trainer

    torch.cuda.set_device(rank)
    ctx = init_zero(120, ep_size=world) if zero else pdist.init(ep_size=world, timeout_s=120)
    try:
        run = GrugRunConfig(model=GrugModelConfig(**CFG), optimizer=GrugMoeAdamHConfig(warmup=0.0),
                            trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=0)))
        tr = Trainer(run, device=f"cuda:{rank}", dist=ctx)
        init = {i.name: tr.store.master_view(i).clone() for i in tr.store.infos}
        tok = torch.randint(0, 4096, (2, 256), generator=torch.Generator().manual_seed(rank)).pin_memory()
        tr.train_step({"tokens": tok})
        torch.cuda.synchronize()
        upd = {i.name: (tr.store.master_view(i) - init[i.name]).cpu().numpy() for i in tr.store.infos}
        return {"upd": upd, "m_numel": tr.opt.m.numel(), "n": tr.store.numel, "rep": tr.store.expert_start}
    finally:
        pdist.shutdown()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero_with_expert_parallelism_on_gpu():
    """ZeRO over the replicated parameters with the experts sharded by expert parallelism (the
    peer-memory exchange): the same update as expert parallelism with replicated optimizer state."""
    a = run_ranks(_ep_rank, 2, True, timeout=300)
    b = run_ranks(_ep_rank, 2, False, timeout=300)
    assert a[0]["m_numel"] == a[0]["rep"] // 2 + (a[0]["n"] - a[0]["rep"])
    for r in range(2):
        num = sum(float(((torch.from_numpy(a[r]["upd"][k]) - torch.from_numpy(v)) ** 2).sum())
                  for k, v in b[r]["upd"].items())
        den = sum(float((torch.from_numpy(v) ** 2).sum()) for v in b[r]["upd"].values())
        assert (num / den) ** 0.5 < 0.05, (r, (num / den) ** 0.5)


def _p2p_rank(rank, world, p2p):
    import os

    os.environ["MXK_ZERO_P2P"] = "1" if p2p else "0"
    out = _rank(rank, world, True)
    return out


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero_peer_memory_matches_nccl():
    """ZeRO's reduce-scatter and all-gather as peer-memory kernels vs NCCL's collectives: the same
    parameter update (fp32 sums of two ranks are exact in either order)."""
    a = run_ranks(_p2p_rank, 2, True, timeout=300)
    b = run_ranks(_p2p_rank, 2, False, timeout=300)
    for r in range(2):
        ua, ub = torch.from_numpy(a[r]["upd"]), torch.from_numpy(b[r]["upd"])
        assert ((ua - ub).norm() / ub.norm()).item() < 1e-2, r
