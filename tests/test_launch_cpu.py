"""Launchers: the tiny-stories corpus -> tokenize -> train -> checkpoint pipeline end to end on CPU,
resume from its checkpoint, the megagpt environment arms, the heuristic and FLOP accounting."""

import json
import math
import os

import pytest

from marin_experiments_b200.experiments import megagpt, tiny_stories
from marin_experiments_b200.executor import Executor


def test_tiny_stories_pipeline(tmp_path, capsys):
    steps = tiny_stories.build_steps(steps=3, batch_size=4)
    res = Executor(str(tmp_path)).run(steps)
    out = capsys.readouterr().out
    assert out.count("[THRUPUT] step=") == 3
    train_dir = res["tiny-stories/tinystories-30m"]
    ck = os.path.join(train_dir, "checkpoints", "step-3", "metadata.json")
    assert json.load(open(ck))["step"] == 3
    metrics = [json.loads(l) for l in open(os.path.join(train_dir, "logs", "tiny-stories-30m-cpu", "metrics.jsonl"))]
    assert [m["step"] for m in metrics] == [1, 2, 3] and all(math.isfinite(m["train/loss"]) for m in metrics)
    # a rerun of the same versions is skipped; the trainer itself resumes from its checkpoint
    from marin_experiments_b200.experiments.common import run_inline
    launch = Executor(str(tmp_path)).instantiate(steps[2])
    import dataclasses
    r = run_inline(dataclasses.replace(launch, steps=4))
    assert r["restored_from"].endswith("step-3") and r["start_step"] == 3 and r["final_step"] == 4


def test_megagpt_arms():
    env = {"SP_HIDDEN": "1536", "SP_EXPERTS": "64", "SP_TOPK": "4", "SP_SEQ": "2048", "SP_EP": "8",
           "SP_BATCH": "256", "SP_STEPS": "10", "SP_SCHEDULE": "constant", "SP_GLOBAL_EVERY": "6"}
    launch, arm = megagpt.make_launch(env)
    m = launch.model.value
    assert (m.hidden_dim, m.num_experts, m.num_experts_per_token, m.intermediate_dim, m.max_seq_len) == \
        (1536, 64, 4, 768, 2048)
    assert m.global_attn_every == 6 and launch.grug_trainer.value.expert_axis_size == 8
    assert launch.optimizer.value.lr_schedule == "constant"
    assert launch.batch_size.value == 256 and launch.steps.value == 10
    from marin_experiments_b200.utils.tracker import THRU  # noqa: F401
    import re
    arm_re = re.compile(r"\[arm\].*?D=(\d+).*?seq=(\d+).*?E=(\d+) k=(\d+).*?batch=(\d+).*?budget=([\d.eE+]+)")
    g = arm_re.search(arm).groups()
    assert g[:5] == ("1536", "2048", "64", "4", "256")
    with pytest.raises(ValueError):
        megagpt.make_launch({"SPARSITY_MODE": "weird"})
    adaptive, _ = megagpt.make_launch({"SPARSITY_MODE": "adaptive", "SP_MIN_K": "1", "SP_COEF": "0.01",
                                       "SP_HIDDEN": "512", "SP_EXPERTS": "32", "SP_TOPK": "8"})
    assert adaptive.model.value.adaptive_routing and adaptive.model.value.sparsity_loss_coef == 0.01


def test_heuristic_values():
    from marin_experiments_b200.optim.heuristic import MoeAdamHHeuristic, build_from_heuristic, compute_tokens_and_batch

    h = MoeAdamHHeuristic()
    assert h.num_layers(1024) == round(1024 / (64 + 40 - 9))
    assert h.kv_heads(16, 4) == 4 and h.kv_heads(12, 4) == 3 and h.kv_heads(6, 4) == 1
    assert h.beta2(131072) == pytest.approx(0.999)
    assert h.beta2(10 ** 9) == 0.95
    tok, b, s = compute_tokens_and_batch(3e18, 1e9, target_steps=1000, seq_len=4096)
    assert tok == pytest.approx(1e9) and b == 256 and s == round(1e9 / (256 * 4096))
    m, o, b, s = build_from_heuristic(budget=1e18, hidden_dim=1024, batch_size=48)
    assert b == 48 and o.learning_rate == pytest.approx(min(0.05, 13 / 3 * o.adam_lr))


def test_flop_accounting():
    from marin_experiments_b200.config import GrugModelConfig
    from marin_experiments_b200.utils.flops import (compute_flops_per_token, fwd_components, lm_flops_per_token,
                                                    training_flops_per_token)

    c = GrugModelConfig(vocab_size=1000, hidden_dim=256, intermediate_dim=128, shared_expert_intermediate_dim=256,
                        num_experts=8, num_experts_per_token=2, num_layers=2, num_heads=4, num_kv_heads=2,
                        head_dim=64, max_seq_len=128)
    f = fwd_components(c)
    assert f["routed_experts"] == 2 * (2 * 3 * 256 * 128 * 2)
    assert f["router_proj"] == 2 * 2 * 256 * 8
    assert f["lm_head"] == 2 * 256 * 1000
    assert f["gated_norms"] == 2 * 2 * (2 * 2 * 256 * 128) + 2 * (2 * 2 * 256 * 128)
    assert compute_flops_per_token(c) == lm_flops_per_token(c) - 2 * 256 * 1000
    assert training_flops_per_token(c, causal=False) == 3 * f["_total"]


@pytest.mark.parametrize("module", ["marin_experiments_b200.experiments.megagpt",
                                    "marin_experiments_b200.experiments.tiny_stories",
                                    "marin_experiments_b200.experiments.delayed_gradient"])
def test_launcher_dry_run_in_fresh_process(module, tmp_path):
    """Every experiment launcher imports and builds its steps with --dry_run (no jobs run)."""
    import subprocess
    import sys

    env = {**os.environ, "MARIN_PREFIX": str(tmp_path), "PYTHONPATH": os.getcwd()}
    r = subprocess.run([sys.executable, "-m", module, "--dry_run"], env=env, capture_output=True, text=True,
                       timeout=300, cwd=str(tmp_path))
    assert r.returncode == 0, r.stderr[-2000:]
    assert "[dry-run]" in r.stdout


def test_delayed_gradient_arms():
    from marin_experiments_b200.experiments import delayed_gradient as dg
    from marin_experiments_b200.optim.delayed import DelayedGrugMoeAdamHConfig, DelayedGrugMuonConfig

    launch, arm = dg.make_launch({"GRUG_OPT": "muon", "GRUG_TAU": "8", "GRUG_CORRECTOR": "dc_asgd_ema",
                                  "GRUG_STEPS": "50", "GRUG_SEQ": "1024"})
    opt = launch.optimizer.value if hasattr(launch.optimizer, "value") else launch.optimizer
    assert isinstance(opt, DelayedGrugMuonConfig) and opt.tau == 8 and opt.corrector == "dc_asgd_ema"
    assert opt.learning_rate == 0.02 and "tau8" in launch.run_id and "corrector=dc_asgd_ema" in arm
    launch2, _ = dg.make_launch({"GRUG_OPT": "adamh", "GRUG_STAGES": "4", "GRUG_TAU": "8", "GRUG_HIDDEN": "768"})
    opt2 = launch2.optimizer.value if hasattr(launch2.optimizer, "value") else launch2.optimizer
    model = launch2.model.value if hasattr(launch2.model, "value") else launch2.model
    assert isinstance(opt2, DelayedGrugMoeAdamHConfig) and opt2.tau == 0 and opt2.num_stages == 4
    assert opt2.num_layers == model.num_layers and model.hidden_dim == 768 and "S4" in launch2.run_id
    with pytest.raises(ValueError):
        dg.make_launch({"GRUG_OPT": "sgd"})
    with pytest.raises(ValueError):
        dg.make_launch({"GRUG_CORRECTOR": "magic"})


@pytest.mark.parametrize("name", ["grug_dp", "adaptive"])
def test_bench_configs_build_and_train(name):
    """The benchmark's smaller configurations are valid models: one training step of a scaled-down copy
    (1 layer, seq 64, vocab 1024) on CPU."""
    import dataclasses
    import sys

    import torch

    sys.path.insert(0, os.getcwd())
    import bench

    from marin_experiments_b200.config import GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    bc = bench.bench_config(name, 8)
    assert bc["scaling"] == "strong" and bc["baseline"] is None
    assert bc["seqs_per_gpu"] * 8 * bc["model"].max_seq_len in (256 * 1024, 128 * 2048)
    cfg = dataclasses.replace(bc["model"], num_layers=1, max_seq_len=64, sliding_window=64, vocab_size=1024)
    run = GrugRunConfig(model=cfg, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=3)))
    tr = Trainer(run, device="cpu")
    tok = torch.randint(0, 1024, (2, 64), generator=torch.Generator().manual_seed(0))
    met = tr.train_step({"tokens": tok})
    assert torch.isfinite(met["train/loss"])
    assert bench.bench_config("megagpt", 1)["micro_batch"] == 8 and bench.bench_config("megagpt", 8)["micro_batch"] == 16
