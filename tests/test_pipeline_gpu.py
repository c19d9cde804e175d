"""Pipeline parallelism on 2 GPUs over NCCL: sync 1F1B and ZB-H1 steps against the unsplit model on
one GPU, and the async no-flush mode."""

import datetime
import os

import pytest
import torch

from mp_util import run_ranks

pytestmark = pytest.mark.gpu

MOE = dict(vocab_size=4096, hidden_dim=256, intermediate_dim=256, shared_expert_intermediate_dim=512, num_experts=8,
           num_experts_per_token=2, num_layers=4, num_heads=4, num_kv_heads=4, head_dim=64, max_seq_len=256,
           sliding_window=256, capacity_factor=4.0)


def _cfg():
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import AdamConfig

    return GrugRunConfig(model=GrugModelConfig(**MOE), optimizer=AdamConfig(warmup=0.0, learning_rate=1e-3),
                         trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=0)))


def _tokens():
    return torch.randint(0, 4096, (8, 256), generator=torch.Generator().manual_seed(7))


def _rank(rank, world, schedule):
    import torch.distributed as tdist

    from marin_experiments_b200.parallel.pipeline import PipelineTrainer, init_topology

    torch.cuda.set_device(rank)
    tdist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        topo = init_topology(world, 1)
        pt = PipelineTrainer(_cfg(), topo, device=f"cuda:{rank}", microbatches=4, schedule=schedule)
        out = pt.train_step({"tokens": _tokens().pin_memory()})
        torch.cuda.synchronize()
        from marin_experiments_b200.ops._ext import check_kernel_errors

        check_kernel_errors()
        g = pt.model.global_name
        return {g(i.name): pt.tr.store.master_view(i).cpu().numpy().copy() for i in pt.tr.store.infos}
    finally:
        tdist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("schedule", ["1f1b", "zb"])
def test_pp2_matches_unsplit(schedule):
    from marin_experiments_b200.train.trainer import Trainer

    res = run_ranks(_rank, 2, schedule, timeout=300)
    ref = Trainer(_cfg(), device="cuda:0", micro_batch=2)
    init = {ref.model.global_name(i.name): ref.store.master_view(i).clone().cpu() for i in ref.store.infos}
    ref.train_step({"tokens": _tokens().pin_memory()})
    want = {ref.model.global_name(i.name): ref.store.master_view(i).cpu() for i in ref.store.infos}
    for part in res.values():
        for name, arr in part.items():
            got = torch.from_numpy(arr)
            upd_ref = want[name] - init[name]
            upd = got - init[name]
            # Adam's first step moves every weight by ~lr * sign(g): compare the updates
            err = ((upd - upd_ref).norm() / upd_ref.norm().clamp_min(1e-12)).item()
            assert err < 0.1, (name, err)


def _rank_pp_ep(rank, world, schedule):
    import torch.distributed as tdist

    from marin_experiments_b200.parallel.pipeline import PipelineTrainer, init_topology

    torch.cuda.set_device(rank)
    tdist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        topo = init_topology(world // 2, 2)
        pt = PipelineTrainer(_cfg(), topo, device=f"cuda:{rank}", microbatches=2, schedule=schedule)
        tok = _tokens()
        local = tok.shape[0] // 2
        pt.train_step({"tokens": tok[topo.e * local:(topo.e + 1) * local].pin_memory()})
        torch.cuda.synchronize()
        from marin_experiments_b200.ops._ext import check_kernel_errors

        check_kernel_errors()
        g = pt.model.global_name
        return {"e": topo.e,
                "params": {g(i.name): pt.tr.store.master_view(i).cpu().numpy().copy() for i in pt.tr.store.infos}}
    finally:
        tdist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("schedule", ["1f1b", "zb"])
def test_pp2_ep2_matches_unsplit(schedule):
    """Pipeline x expert parallelism on 4 GPUs (2 stages x 2 expert ranks, the token exchange over
    peer memory) against the unsplit model on one GPU."""
    from marin_experiments_b200.train.trainer import Trainer

    res = run_ranks(_rank_pp_ep, 4, schedule, timeout=300)
    ref = Trainer(_cfg(), device="cuda:0", micro_batch=2)
    init = {ref.model.global_name(i.name): ref.store.master_view(i).clone().cpu() for i in ref.store.infos}
    ref.train_step({"tokens": _tokens().pin_memory()})
    want = {ref.model.global_name(i.name): ref.store.master_view(i).cpu() for i in ref.store.infos}
    for part in res.values():
        for name, arr in part["params"].items():
            got = torch.from_numpy(arr)
            w, i0 = want[name], init[name]
            if got.dim() == 3 and ".mlp.w_" in name and got.shape[0] != w.shape[0]:
                n = got.shape[0]
                w, i0 = w[part["e"] * n:(part["e"] + 1) * n], i0[part["e"] * n:(part["e"] + 1) * n]
            upd_ref, upd = w - i0, got - i0
            err = ((upd - upd_ref).norm() / upd_ref.norm().clamp_min(1e-12)).item()
            assert err < 0.1, (name, err)
