"""Throughput lines and their monitor parser, the JSONL tracker, the step watchdog, and the
active-expert curriculum."""

import io
import json
import time

import torch

from marin_experiments_b200.config import GrugModelConfig
from marin_experiments_b200.train.curriculum import active_k_at, parse_curriculum, set_active_k
from marin_experiments_b200.utils.tracker import JsonlTracker, ThroughputHook, Watchdog, parse_thruput

CFG = GrugModelConfig(vocab_size=512, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128,
                      num_experts=8, num_experts_per_token=2, num_layers=2, num_heads=2, num_kv_heads=2, head_dim=32,
                      max_seq_len=64, sliding_window=64)


def test_thruput_roundtrip():
    buf = io.StringIO()
    hook = ThroughputHook(CFG, n_gpus=1, stream=buf)
    for s in range(1, 11):
        hook(None, {"step": s, "step_duration": 0.5, "tokens": 1000, "batch_size": 4})
    r = parse_thruput(buf.getvalue(), warmup=5)
    assert r["n"] == 6 and r["tok_s"] == 2000.0 and r["mfu"] is not None


def test_jsonl_tracker(tmp_path):
    t = JsonlTracker(str(tmp_path), "run", {"a": 1})
    t.log({"loss": torch.tensor(2.5)}, step=3)
    t.log_summary({"final": 1})
    t.finish()
    line = json.loads(open(tmp_path / "run" / "metrics.jsonl").read().splitlines()[0])
    assert line == {"step": 3, "loss": 2.5}


def test_watchdog_fires_and_kicks():
    fired = []
    wd = Watchdog(0.2, on_timeout=fired.append, poll_s=0.02, stream=io.StringIO()).start()
    for _ in range(10):
        time.sleep(0.05)
        wd.kick()
    assert not fired
    time.sleep(0.5)
    wd.stop()
    assert fired and fired[0] >= 0.2


def test_curriculum_schedule_and_swap():
    sched = parse_curriculum("1:0.25,2:0.25,4:0.5", 100)
    assert sched == ((1, 25), (2, 50), (4, 100))
    assert [active_k_at(sched, s) for s in (0, 24, 25, 60, 150)] == [1, 1, 2, 4, 4]
    from marin_experiments_b200.models.grug import Transformer

    m = Transformer(CFG)
    m.init_weights(0)
    assert set_active_k(m, 4)
    ks = {mod.cfg.num_experts_per_token for mod in m.modules() if getattr(mod, "cfg", None) is not None}
    assert ks == {4}
    assert not set_active_k(m, 4)
    tok = torch.randint(0, 512, (2, 64))
    loss, met = m.next_token_loss(tok)
    assert torch.isfinite(loss)


def test_router_histogram_coarsening_and_layer_metrics():
    import torch

    from marin_experiments_b200.utils.tracker import coarsen_counts, router_layer_metrics

    assert coarsen_counts([1, 2, 3]) == [1.0, 2.0, 3.0]
    big = torch.arange(1024, dtype=torch.float32)
    h = coarsen_counts(big)
    assert len(h) == 256 and h[0] == 0 + 1 + 2 + 3 and sum(h) == float(big.sum())
    odd = coarsen_counts(list(range(600)), max_buckets=256)  # groups of 3, last padded
    assert len(odd) == 200 and sum(odd) == sum(range(600))
    m = router_layer_metrics({"routing_entropy_per_layer": torch.tensor([1.5, 2.0]),
                              "routing_counts_per_layer": torch.tensor([[3, 1], [2, 2]])})
    assert m["train/router/layer_1/routing_entropy"] == 2.0
    assert m["train/router/layer_0/routing_hist"] == [3.0, 1.0]


def test_wandb_tracker_with_fake_module(tmp_path, monkeypatch):
    import json
    import sys
    import types

    import pytest

    from marin_experiments_b200.utils import tracker as T

    calls = {}

    class Run:
        def __init__(self):
            self.summary, self.logged, self.finished = {}, [], False

        def log(self, m, step):
            self.logged.append((step, m))

        def finish(self):
            self.finished = True

    def init(**kw):
        calls["init"] = kw
        calls["run"] = Run()
        return calls["run"]

    monkeypatch.setitem(sys.modules, "wandb", types.SimpleNamespace(init=init))
    monkeypatch.setenv("WANDB_PROJECT", "proj")
    monkeypatch.setenv("WANDB_TAGS", "a,b")
    monkeypatch.setenv("WANDB_MODE", "offline")
    t = T.make_tracker("wandb", str(tmp_path), "run-1", {"lr": 0.1})
    t.log({"train/loss": 2.5}, 3)
    t.log_summary({"final": 1.0})
    t.finish()
    kw = calls["init"]
    assert kw["project"] == "proj" and kw["tags"] == ["a", "b"] and kw["mode"] == "offline" and kw["name"] == "run-1"
    assert calls["run"].logged == [(3, {"train/loss": 2.5})] and calls["run"].summary == {"final": 1.0}
    assert calls["run"].finished
    line = json.loads(open(tmp_path / "run-1" / "metrics.jsonl").read().splitlines()[0])
    assert line == {"step": 3, "train/loss": 2.5}  # the JSONL copy is kept
    monkeypatch.setitem(sys.modules, "wandb", None)  # not installed: a clear error, not a silent no-op
    with pytest.raises(ImportError, match="needs the wandb package"):
        T.make_tracker("wandb", str(tmp_path), "run-2")
    assert isinstance(T.make_tracker("wandb", str(tmp_path), "run-3", rank=1), T.NoopTracker)
