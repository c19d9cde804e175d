"""Pipeline parallelism on gloo ranks: schedules, and gradient-exact sync steps (GPipe, 1F1B,
ZB-H1; pure PP and PP x EP) against the unsplit single-process model; the async no-flush mode."""

import pytest
import torch

from marin_experiments_b200.parallel import schedules as S
from mp_util import run_ranks

MOE = dict(vocab_size=512, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128, num_experts=4,
           num_experts_per_token=2, num_layers=4, num_heads=2, num_kv_heads=2, head_dim=32, max_seq_len=32,
           sliding_window=32, capacity_factor=8.0, router_z_loss_coef=0.01)


def _run_cfg(opt="adamh"):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import AdamConfig, GrugMoeAdamHConfig

    o = GrugMoeAdamHConfig(warmup=0.0, max_grad_norm=0.5) if opt == "adamh" else AdamConfig(warmup=0.0)
    return GrugRunConfig(model=GrugModelConfig(**MOE), optimizer=o,
                         trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=0),
                                                   z_loss_weight=1e-3))


def _batch(b=8):
    return torch.randint(0, 512, (b, 32), generator=torch.Generator().manual_seed(5))


def test_schedules_valid_and_bubbles():
    for P, M in ((2, 2), (2, 5), (4, 4), (4, 8), (3, 7)):
        for name, fn in S.SCHEDULES.items():
            S.validate(fn(P, M), M)
    g = S.simulate(S.gpipe(4, 8), 1, 2)
    o = S.simulate(S.one_f_one_b(4, 8), 1, 2)
    z = S.simulate(S.zb_h1(4, 8), 1, 1, 1)
    assert g["makespan"] == o["makespan"] and z["bubble"] < o["bubble"]
    from marin_experiments_b200.parallel.pipeline import async_stage_delay, stage_layers

    assert [async_stage_delay(4, s) for s in range(4)] == [6, 4, 2, 0]
    assert list(stage_layers(24, 4, 1)) == list(range(6, 12))
    with pytest.raises(ValueError):
        stage_layers(10, 4, 0)


def _oracle(micro):
    from marin_experiments_b200.train.trainer import Trainer

    tr = Trainer(_run_cfg(), device="cpu", micro_batch=micro)
    tr.train_step({"tokens": _batch()})
    gname = tr.model.global_name
    return {gname(i.name): tr.store.master_view(i).clone() for i in tr.store.infos}


def _pp_rank(rank, world, pp, ep, schedule, zero=False):
    import torch.distributed as tdist

    from marin_experiments_b200.parallel.pipeline import PipelineTrainer, init_topology

    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        topo = init_topology(pp, ep)
        pt = PipelineTrainer(_run_cfg(), topo, device="cpu", microbatches=2, schedule=schedule, zero=zero)
        tok = _batch()
        local = tok.shape[0] // ep
        out = pt.train_step({"tokens": tok[topo.e * local:(topo.e + 1) * local]})
        gname = pt.model.global_name
        params = {gname(i.name): pt.tr.store.master_view(i).numpy().copy() for i in pt.tr.store.infos}
        return {"stage": topo.stage, "e": topo.e, "params": params,
                "loss": float(out["train/cross_entropy_loss"]) if out else None}
    finally:
        tdist.destroy_process_group()


def _check(res, oracle, ep):
    for r, v in res.items():
        for name, arr in v["params"].items():
            want = oracle[name]
            got = torch.from_numpy(arr)
            if ep > 1 and got.dim() == 3 and ".mlp.w_" in name:
                n = got.shape[0]
                want = want[v["e"] * n:(v["e"] + 1) * n]
            assert torch.allclose(got, want, atol=2e-5, rtol=1e-4), (r, name, (got - want).abs().max())


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b", "zb"])
def test_pp2_sync_matches_unsplit(schedule):
    res = run_ranks(_pp_rank, 2, 2, 1, schedule)
    _check(res, _oracle(micro=4), 1)


def test_pp2_ep2_sync_matches_unsplit():
    res = run_ranks(_pp_rank, 4, 2, 2, "1f1b")
    _check(res, _oracle(micro=2), 2)


def test_pp2_ep2_zero_matches_unsplit():
    """Pipeline x expert parallelism x ZeRO: each stage shards its replicated parameters' optimizer
    state over its two ranks; the step equals the unsplit model's."""
    res = run_ranks(_pp_rank, 4, 2, 2, "zb", True)
    _check(res, _oracle(micro=2), 2)


def _async_rank(rank, world):
    import torch.distributed as tdist

    from marin_experiments_b200.parallel.pipeline import PipelineTrainer, init_topology

    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        topo = init_topology(world, 1)
        pt = PipelineTrainer(_run_cfg("adam"), topo, device="cpu", microbatches=1, mode="async")
        g = torch.Generator().manual_seed(3)
        mbs = ({"tokens": torch.randint(0, 512, (2, 32), generator=g)} for _ in range(6))
        losses = pt.run_async(mbs, 6)
        return {"stage": topo.stage, "losses": losses, "steps": pt.tr.step}
    finally:
        tdist.destroy_process_group()


def test_async_no_flush():
    res = run_ranks(_async_rank, 2)
    last = [v for v in res.values() if v["stage"] == 1][0]
    assert len(last["losses"]) == 6 and all(l == l for l in last["losses"])
    assert all(v["steps"] == 6 for v in res.values())


def test_pipeline_entry_env_aliases(monkeypatch):
    from marin_experiments_b200.parallel import pipeline_entry as pe

    for k in list(pe._ALIASES) + list(pe._ALIASES.values()):
        monkeypatch.delenv(k, raising=False)
    base = pe._config(False, 2, 0).model
    assert base.hidden_dim == 1536 and base.num_experts == 64
    monkeypatch.setenv("MOE_PP_HIDDEN", "768")
    monkeypatch.setenv("MOE_PP_EXPERTS", "16")
    monkeypatch.setenv("MOE_PP_EPT", "2")
    monkeypatch.setenv("MOE_PP_LAYERS", "4")
    monkeypatch.setenv("SP_SEQ", "512")  # the SP_* name wins over its alias
    monkeypatch.setenv("MOE_PP_SEQ", "64")
    m = pe._config(True, 2, 0).model
    assert (m.hidden_dim, m.num_heads, m.num_experts, m.num_experts_per_token, m.num_layers, m.max_seq_len) == \
        (768, 8, 16, 2, 4, 512)
    monkeypatch.setenv("MOE_PP_STAGE", "4")
    assert pe._env("SP_PP", "1") == "4"


def _pp_transport_rank(rank, world, transport):
    import os

    os.environ["SP_PP_TRANSPORT"] = transport
    return _pp_rank(rank, world, 2, 1, "1f1b")


def test_pp_null_transport():
    """The null transport (zeros at the stage boundary, no traffic) runs the same steps to a finite
    loss that differs from the real transfer's."""
    p2p = run_ranks(_pp_rank, 2, 2, 1, "1f1b", timeout=120)
    null = run_ranks(_pp_transport_rank, 2, "null", timeout=120)
    last = max(p2p, key=lambda r: p2p[r]["stage"])
    assert null[last]["loss"] is not None and null[last]["loss"] == null[last]["loss"]
    assert null[last]["loss"] != p2p[last]["loss"]


def test_null_transport_reference_switch(monkeypatch):
    """The reference benchmark's MOE_PP_NULL_XPORT=1 selects the null stage transport; an explicit
    SP_PP_TRANSPORT wins over it."""
    from marin_experiments_b200.parallel.pipeline import stage_transport

    monkeypatch.delenv("SP_PP_TRANSPORT", raising=False)
    monkeypatch.delenv("MOE_PP_NULL_XPORT", raising=False)
    assert stage_transport() == "p2p"
    monkeypatch.setenv("MOE_PP_NULL_XPORT", "1")
    assert stage_transport() == "null"
    monkeypatch.setenv("SP_PP_TRANSPORT", "p2p")
    assert stage_transport() == "p2p"
    monkeypatch.delenv("SP_PP_TRANSPORT")
    monkeypatch.setenv("MOE_PP_NULL_XPORT", "0")
    assert stage_transport() == "p2p"


def test_max_inflight_microbatches():
    """Expert-parallel buffers per in-flight microbatch: GPipe holds every microbatch, 1F1B at most P."""
    from marin_experiments_b200.parallel.pipeline import max_inflight

    assert max_inflight("gpipe", 4, 16) == 16
    assert max_inflight("1f1b", 4, 16) == 4
    assert max_inflight("zb", 4, 16) <= 4
    assert max_inflight("1f1b", 4, 16, mode="async") == 4
    assert max_inflight("1f1b", 1, 8) == 1


def _p2p_rank(rank, world):
    import torch.distributed as tdist

    from marin_experiments_b200.benchmarks.p2p_probe import probe

    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        return probe((0.25, 1), iters=2)
    finally:
        tdist.destroy_process_group()


def test_p2p_ring_probe():
    res = run_ranks(_p2p_rank, 3, timeout=120)
    rows = res[0]
    assert [r["mb"] for r in rows] == [0.25, 1] and all(r["gbs_per_direction"] > 0 for r in rows)
    assert rows[0]["ms"] == res[1][0]["ms"]  # max over ranks, the same on every rank
