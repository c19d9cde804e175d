"""ZeRO-2 data parallelism on gloo ranks: sharded optimizer state gives the same parameters as
replicated data parallelism, and a sharded checkpoint round-trips."""

import torch

from mp_util import run_ranks

CFG = dict(vocab_size=512, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128, num_experts=4,
           num_experts_per_token=2, num_layers=2, num_heads=2, num_kv_heads=2, head_dim=32, max_seq_len=32,
           sliding_window=32, capacity_factor=8.0)


def _trainer(ctx, opt="adamh"):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import AdamConfig, GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    if opt == "muon":
        from marin_experiments_b200.optim.configs import MuonConfig

        o = MuonConfig(warmup=0.0, weight_decay=0.1)
    else:
        o = GrugMoeAdamHConfig(warmup=0.0, max_grad_norm=0.3) if opt == "adamh" else \
            AdamConfig(warmup=0.0, weight_decay=0.1)
    run = GrugRunConfig(model=GrugModelConfig(**CFG), optimizer=o,
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=0)))
    return Trainer(run, device="cpu", dist=ctx)


def _rank(rank, world, zero, opt, ckpt, steps=2):
    import torch.distributed as tdist

    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.parallel.fsdp import init_zero

    ctx = init_zero(120) if zero else pdist.init(ep_size=1, timeout_s=120)
    try:
        tr = _trainer(ctx, opt)
        g = torch.Generator().manual_seed(11 + rank)
        for _ in range(steps):
            tr.train_step({"tokens": torch.randint(0, 512, (2, 32), generator=g)})
        out = {"master": tr.store.master.numpy().copy()}
        if ckpt:
            from marin_experiments_b200.train.checkpoint import load_checkpoint, save_checkpoint

            save_checkpoint(tr, ckpt)
            tdist.barrier()
            fresh = _trainer(ctx, opt)
            load_checkpoint(fresh, ckpt)
            out["m_equal"] = bool(torch.equal(fresh.opt.m, tr.opt.m) and torch.equal(fresh.opt.v, tr.opt.v))
            out["p_equal"] = bool(torch.equal(fresh.store.master, tr.store.master))
            out["m_numel"] = tr.opt.m.numel()
            out["store"] = tr.store.numel
        return out
    finally:
        pdist.shutdown()


def test_zero_matches_replicated_dp_adamh():
    a = run_ranks(_rank, 2, True, "adamh", None)
    b = run_ranks(_rank, 2, False, "adamh", None)
    for r in range(2):
        assert torch.allclose(torch.from_numpy(a[r]["master"]), torch.from_numpy(b[r]["master"]), atol=1e-5, rtol=1e-4)
    assert torch.equal(torch.from_numpy(a[0]["master"]), torch.from_numpy(a[1]["master"]))


def test_zero_adamw_checkpoint_roundtrip(tmp_path):
    a = run_ranks(_rank, 2, True, "adam", str(tmp_path / "step-2"))
    b = run_ranks(_rank, 2, False, "adam", None)
    for r in range(2):
        assert a[r]["m_equal"] and a[r]["p_equal"]
        assert a[r]["m_numel"] * 2 == a[r]["store"]
        assert torch.allclose(torch.from_numpy(a[r]["master"]), torch.from_numpy(b[r]["master"]), atol=1e-6)


def _maxdiff(opt="adamh", steps=2):
    a = run_ranks(_rank, 2, True, opt, None, steps)
    b = run_ranks(_rank, 2, False, opt, None, steps)
    d = (torch.from_numpy(a[0]["master"]) - torch.from_numpy(b[0]["master"])).abs()
    return d.max().item(), d.argmax().item(), (d > 1e-5).sum().item()


def _dp_rank(rank, world, ep):
    from marin_experiments_b200.parallel import dist as pdist

    ctx = pdist.init(ep_size=ep, timeout_s=120)
    try:
        tr = _trainer(ctx, "adam")
        tok = torch.randint(0, 512, (world * 2, 32), generator=torch.Generator().manual_seed(21))
        tr.train_step({"tokens": tok[rank * 2:(rank + 1) * 2]})
        g = tr.model.global_name
        return {"e": ctx.ep_rank, "p": {g(i.name): tr.store.master_view(i).numpy().copy() for i in tr.store.infos}}
    finally:
        pdist.shutdown()


def test_data_and_expert_parallel_match_single_process():
    single = _trainer(None, "adam")
    single.micro_batch = 2
    tok = torch.randint(0, 512, (8, 32), generator=torch.Generator().manual_seed(21))
    single.train_step({"tokens": tok})
    want = {i.name: single.store.master_view(i) for i in single.store.infos}
    for world, ep in ((4, 1), (4, 2)):
        res = run_ranks(_dp_rank, world, ep)
        for r, v in res.items():
            for name, arr in v["p"].items():
                w = want[name]
                got = torch.from_numpy(arr)
                if got.shape != w.shape:  # expert shard
                    n = got.shape[0]
                    w = w[v["e"] * n:(v["e"] + 1) * n]
                assert torch.allclose(got, w, atol=1e-6, rtol=1e-5), (world, ep, r, name)


def _ep_rank(rank, world, zero, ckpt):
    """Expert parallelism (EP = world) with or without ZeRO over the replicated parameters."""
    import torch.distributed as tdist

    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.parallel.fsdp import init_zero

    ctx = init_zero(120, ep_size=world) if zero else pdist.init(ep_size=world, timeout_s=120)
    try:
        tr = _trainer(ctx, "adamh")
        g = torch.Generator().manual_seed(21 + rank)
        for _ in range(2):
            tr.train_step({"tokens": torch.randint(0, 512, (2, 32), generator=g)})
        out = {"params": {i.name: tr.store.master_view(i).numpy().copy() for i in tr.store.infos},
               "m_numel": tr.opt.m.numel(), "store": tr.store.numel,
               "expert_start": tr.store.expert_start}
        if ckpt:
            from marin_experiments_b200.train.checkpoint import load_checkpoint, save_checkpoint

            save_checkpoint(tr, ckpt)
            tdist.barrier()
            fresh = _trainer(ctx, "adamh")
            load_checkpoint(fresh, ckpt)
            out["m_equal"] = bool(torch.equal(fresh.opt.m, tr.opt.m) and torch.equal(fresh.opt.v, tr.opt.v))
            out["p_equal"] = bool(torch.equal(fresh.store.master, tr.store.master))
        return out
    finally:
        pdist.shutdown()


def test_zero_with_expert_parallelism(tmp_path):
    """ZeRO over the replicated parameters + experts sharded by expert parallelism: the same weights
    as expert parallelism with replicated optimizer state; the replicated moments are split over the
    ranks and each rank keeps its own experts' moments; the sharded checkpoint round-trips."""
    a = run_ranks(_ep_rank, 2, True, str(tmp_path / "step-2"))
    b = run_ranks(_ep_rank, 2, False, None)
    for r in range(2):
        assert a[r]["m_equal"] and a[r]["p_equal"]
        rep, n = a[r]["expert_start"], a[r]["store"]
        assert rep is not None and a[r]["m_numel"] == rep // 2 + (n - rep)
        for name, want in b[r]["params"].items():
            assert torch.allclose(torch.from_numpy(a[r]["params"][name]), torch.from_numpy(want), atol=1e-5,
                                  rtol=1e-4), name


def test_muon_bounds_move_past_matrices():
    from marin_experiments_b200.parallel.fsdp import muon_bounds

    # spans [0,40) [40,200) [200,256); world 4, equal ranges of 64
    assert muon_bounds([(0, 40), (40, 200), (200, 256)], 256, 4) == [0, 200, 200, 200, 256]
    assert muon_bounds([(10, 20)], 256, 4) == [0, 64, 128, 192, 256]
    assert muon_bounds([(60, 70), (120, 130)], 256, 4) == [0, 70, 130, 192, 256]


def _muon_rank(rank, world, zero, steps=3):
    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.parallel.fsdp import init_zero

    ctx = init_zero(120) if zero else pdist.init(ep_size=1, timeout_s=120)
    try:
        tr = _trainer(ctx, "muon")
        g = torch.Generator().manual_seed(11 + rank)
        for _ in range(steps):
            tr.train_step({"tokens": torch.randint(0, 512, (2, 32), generator=g)})
        inner = getattr(tr.opt, "inner", tr.opt)
        b = getattr(ctx, "_bounds", None)
        crossing = b is not None and any(b[r] != r * (ctx._end // world) for r in range(1, world))
        return {"master": tr.store.master.numpy().copy(), "owned": len(inner.muon_owned),
                "all": len(inner.muon_infos), "m_numel": inner.m.numel(), "crossing": crossing}
    finally:
        pdist.shutdown()


def test_zero_muon_matches_replicated_dp():
    """Muon under ZeRO: each matrix is orthogonalised whole by one owner (some cross the equal
    reduce-scatter boundaries), and the parameters equal replicated data parallelism's."""
    for world in (2, 3):
        a = run_ranks(_muon_rank, world, True)
        b = run_ranks(_muon_rank, world, False)
        assert any(a[r]["crossing"] for r in range(world))
        assert sum(a[r]["owned"] for r in range(world)) == a[0]["all"]
        for r in range(world):  # the ZeRO store is padded to a multiple of 64 x world elements
            n = min(a[r]["master"].size, b[r]["master"].size)
            assert torch.allclose(torch.from_numpy(a[r]["master"][:n]), torch.from_numpy(b[r]["master"][:n]),
                                  atol=1e-5, rtol=1e-4)
        assert all(torch.equal(torch.from_numpy(a[0]["master"]), torch.from_numpy(a[r]["master"]))
                   for r in range(world))
