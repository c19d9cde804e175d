"""Watch statistics, the step profiler hook and NVTX ranges on the tiny dense CPU configuration."""

import math
import os

import torch

from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
from marin_experiments_b200.optim import AdamConfig
from marin_experiments_b200.train.trainer import Trainer
from marin_experiments_b200.utils.profiling import ProfilerHook, nvtx_range, watch_stats

TINY = GrugModelConfig(vocab_size=1024, hidden_dim=128, intermediate_dim=256, num_experts=0, num_layers=2,
                       num_heads=4, num_kv_heads=4, head_dim=32, max_seq_len=64, sliding_window=64,
                       gated_norm=False, qk_norm=False, xsa=False, head_gate=False, shared_expert_intermediate_dim=0)


def _trainer(steps=10):
    run = GrugRunConfig(model=TINY, optimizer=AdamConfig(learning_rate=3e-4, warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=steps, seed=0)))
    return Trainer(run, device="cpu")


def _batches(n):
    g = torch.Generator().manual_seed(0)
    return [{"tokens": torch.randint(0, 1024, (4, 64), generator=g)} for _ in range(n)]


def test_watch_stats_norms():
    tr = _trainer()
    st = tr.store
    st.grad.normal_(0, 1e-3, generator=torch.Generator().manual_seed(1))
    w = watch_stats(st, per_param=True, hist_bins=16)
    assert math.isclose(w["watch/grad_norm/total"], float(st.grad.norm()), rel_tol=1e-4)
    assert math.isclose(w["watch/param_norm/total"], float(st.master.norm()), rel_tol=1e-4)
    info = st.infos[3]
    g = st.grad[info.offset: info.offset + info.numel]
    assert math.isclose(w[f"watch/grad_norm/{info.name}"], float(g.norm()), rel_tol=1e-4)
    kinds = [k.split("/")[-1] for k in w if k.startswith("watch/grad_norm/") and "blocks" not in k]
    assert "attn.w_qkv" in kinds and "total" in kinds
    assert all(not any(part.isdigit() for part in k.split(".")) for k in kinds)  # layer indices folded
    assert len(w["watch/grad_hist"]) == 16 and abs(sum(w["watch/grad_hist"]) - st.grad.numel()) < 1.0


def test_watch_in_train_step_and_profiler_hook(tmp_path):
    tr = _trainer(steps=6)
    tr.watch_every = 2
    prof = ProfilerHook(str(tmp_path / "profiler"), start_step=2, num_steps=2)
    seen = []
    last = tr.fit(iter(_batches(6)), 6, hooks=[prof, lambda t, info: seen.append(info)], pre_hooks=[prof])
    assert last["step"] == 6 and prof.done and prof.prof is None
    assert os.path.exists(tmp_path / "profiler" / "trace.json")
    text = open(tmp_path / "profiler" / "breakdown.md").read()
    assert text.startswith("steps 2..3") and "ms/step" in text
    has = [("watch/grad_norm/total" in i["metrics"]) for i in seen]
    # train_step computes watch stats when step % 2 == 0 before its increment: steps 0, 2, 4
    assert has == [True, False, True, False, True, False]
    assert all(i["metrics"]["watch/grad_norm/total"] > 0 for i, h in zip(seen, has) if h)


def test_nvtx_range_is_a_noop_without_cuda(monkeypatch):
    monkeypatch.setenv("MXK_NVTX", "1")
    with nvtx_range("x"):
        y = 1
    assert y == 1


def _watch_rank(rank, world):
    import datetime
    from types import SimpleNamespace

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # two parameters: a replicated one (same values on every rank) and an expert shard (per rank)
        grad = torch.tensor([3.0, 4.0] + [float(rank + 1)] * 4)
        master = torch.ones(6)
        infos = [SimpleNamespace(name="blocks.0.attn.w_o", offset=0, numel=2, sharded_over=None),
                 SimpleNamespace(name="blocks.0.mlp.w_down", offset=2, numel=4, sharded_over="expert")]
        store = SimpleNamespace(infos=infos, grad=grad, master=master)
        return watch_stats(store, ep_group=dist.group.WORLD)
    finally:
        dist.destroy_process_group()


def test_watch_stats_sums_expert_shards_over_ranks():
    from tests.mp_util import run_ranks

    res = run_ranks(_watch_rank, 2)
    for r in (0, 1):
        w = res[r]
        assert math.isclose(w["watch/grad_norm/attn.w_o"], 5.0)  # replicated: not summed
        assert math.isclose(w["watch/grad_norm/mlp.w_down"], math.sqrt(4 * 1 + 4 * 4))  # both ranks' shards
        assert math.isclose(w["watch/grad_norm/total"], math.sqrt(25 + 20))


def test_tracker_gets_throughput_loading_and_hook_time(tmp_path):
    import io
    import json

    from marin_experiments_b200.utils.tracker import JsonlTracker, ThroughputHook

    tr = _trainer(steps=3)
    trk = JsonlTracker(str(tmp_path), "run")
    thr = ThroughputHook(TINY, 1, stream=io.StringIO())
    tr.fit(iter(_batches(3)), 3, hooks=[thr], tracker=trk, log_every=1)
    trk.finish()
    rows = [json.loads(x) for x in open(tmp_path / "run" / "metrics.jsonl")]
    assert len(rows) == 3
    for r in rows:
        assert r["throughput/tokens_per_second"] > 0 and r["throughput/loading_time"] >= 0
        assert r["throughput/hook_time"] >= 0 and r["throughput/step_duration"] > 0 and "train/loss" in r
