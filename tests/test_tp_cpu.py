"""Tensor parallelism (TP = 2, gloo): sharded heads / MLP units give the unsplit model's loss and,
after an AdamH step with global clipping, its parameters."""

import torch

from mp_util import run_ranks

CFG = dict(vocab_size=256, hidden_dim=64, intermediate_dim=256, shared_expert_intermediate_dim=256, num_experts=4,
           num_experts_per_token=2, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=16, max_seq_len=32,
           sliding_window=32, capacity_factor=8.0)


def _run(tp=None):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    run = GrugRunConfig(model=GrugModelConfig(**CFG), optimizer=GrugMoeAdamHConfig(warmup=0.0, max_grad_norm=0.2),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=0)))
    tr = Trainer(run, device="cpu", model_kwargs={} if tp is None else {"tp": tp})
    if tp is not None:
        from marin_experiments_b200.parallel.tp import setup_tp_optimizer

        setup_tp_optimizer(tr, tp)
    return tr


def _rank(rank, world):
    import torch.distributed as tdist

    from marin_experiments_b200.parallel.tp import TPInfo

    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tr = _run(TPInfo(rank, world, tdist.group.WORLD))
        tok = torch.randint(0, 256, (2, 32), generator=torch.Generator().manual_seed(4))
        met = tr.train_step({"tokens": tok})
        return {"loss": float(met["train/loss"]),
                "p": {i.name: tr.store.master_view(i).numpy().copy() for i in tr.store.infos}}
    finally:
        tdist.destroy_process_group()


def test_tp2_matches_unsplit():
    from marin_experiments_b200.models.grug import Attention, DenseMLP
    from marin_experiments_b200.parallel.tp import TPInfo, shard

    res = run_ranks(_rank, 2)
    ref = _run()
    tok = torch.randint(0, 256, (2, 32), generator=torch.Generator().manual_seed(4))
    want_loss = float(ref.train_step({"tokens": tok})["train/loss"])
    assert abs(res[0]["loss"] - want_loss) < 1e-4 and abs(res[1]["loss"] - want_loss) < 1e-4
    mods = dict(ref.model.named_modules())
    for r in (0, 1):
        for name, arr in res[r]["p"].items():
            got = torch.from_numpy(arr)
            full = ref.store.master_view(ref.store.by_name[name])
            mod = mods[name.rsplit(".", 1)[0] if "." in name else ""]
            leaf = name.rsplit(".", 1)[-1]
            if isinstance(mod, (Attention, DenseMLP)) and leaf in mod.tp_sharded_params:
                full = shard(leaf, full, mod, TPInfo(r, 2))
            assert torch.allclose(got, full, atol=2e-5, rtol=1e-4), (r, name, (got - full).abs().max())
