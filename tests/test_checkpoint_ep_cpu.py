"""Expert-parallel checkpoints on two gloo ranks: each rank writes its expert shard, rank 0 the
replicated leaves; a single process (ep_size 1) restores the full state by resharding."""

import os

import torch

from mp_util import run_ranks

MOE = dict(vocab_size=512, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128, num_experts=4,
           num_experts_per_token=2, num_layers=2, num_heads=2, num_kv_heads=2, head_dim=32, max_seq_len=64,
           sliding_window=64, capacity_factor=2.0)


def _make(dist_ctx=None, seed=0):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    run = GrugRunConfig(model=GrugModelConfig(**MOE), optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=seed)))
    return Trainer(run, device="cpu", dist=dist_ctx)


def _rank(rank, world, path):
    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.train.checkpoint import save_checkpoint

    ctx = pdist.init(ep_size=world, timeout_s=120)
    try:
        tr = _make(ctx)
        g = torch.Generator().manual_seed(rank)
        for _ in range(2):
            tr.train_step({"tokens": torch.randint(0, 512, (2, 64), generator=g)})
        save_checkpoint(tr, path)
        return {i.name: tr.store.master_view(i).numpy().copy() for i in tr.store.infos}
    finally:
        pdist.shutdown()


def test_ep_checkpoint_reshard(tmp_path):
    from marin_experiments_b200.train.checkpoint import load_checkpoint

    path = str(tmp_path / "step-2")
    res = run_ranks(_rank, 2, path)
    files = [f for dp, _, fs in os.walk(path) for f in fs]
    assert any(".e0-2.bin" in f for f in files) and any(".e2-4.bin" in f for f in files)
    single = _make(seed=7)
    load_checkpoint(single, path)
    assert single.step == 2
    for info in single.store.infos:
        got = single.store.master_view(info)
        if info.ndim == 3 and ".mlp.w_" in info.name:
            want = torch.cat([torch.from_numpy(res[0][info.name]), torch.from_numpy(res[1][info.name])])
        else:
            want = torch.from_numpy(res[0][info.name])
        assert torch.equal(got, want), info.name
