"""Failure detection on the host: the NaN stop of the training loop, and a data-parallel job that
loses a rank between steps and resumes from its last checkpoint (gloo ranks on CPU).

Failures are made on the host only: a poisoned weight, a rank that returns without joining the
next step. The surviving rank learns of the loss through a short process-group timeout on its next
collective."""

import os

import pytest
import torch

from mp_util import run_ranks

MOE = dict(vocab_size=512, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128, num_experts=4,
           num_experts_per_token=2, num_layers=2, num_heads=2, num_kv_heads=2, head_dim=32, max_seq_len=64,
           sliding_window=64, capacity_factor=2.0)


def _make(dist_ctx=None, seed=0, steps=10):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    run = GrugRunConfig(model=GrugModelConfig(**MOE), optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=steps, seed=seed)))
    return Trainer(run, device="cpu", dist=dist_ctx)


class _Loader:
    """Deterministic per-(rank, step) batches, so a resumed run sees the same data as an unbroken one."""

    def __init__(self, rank, start=0):
        self.rank, self.step = rank, start

    def __iter__(self):
        return self

    def __next__(self):
        g = torch.Generator().manual_seed(1000 * self.rank + self.step)
        self.step += 1
        return {"tokens": torch.randint(0, 512, (2, 64), generator=g)}


class _Poison:
    """Pre-step hook: at ``step`` overwrite one weight with NaN."""

    def __init__(self, step):
        self.at = step

    def before_step(self, tr):
        if tr.step == self.at:
            with torch.no_grad():
                tr.store.master[:16] = float("nan")
                tr.store.sync_compute()


def test_nan_loss_stops_the_loop_before_checkpointing(tmp_path):
    from marin_experiments_b200.config import CheckpointerConfig
    from marin_experiments_b200.train.checkpoint import Checkpointer, scan_checkpoint_root

    tr = _make(steps=6)
    ck = Checkpointer(CheckpointerConfig(base_path=str(tmp_path), save_interval_s=1e9, keep=[{"every": 1}]),
                      background=False)
    with pytest.raises(FloatingPointError, match="at step 4"):  # reported after the step counter advanced
        tr.fit(_Loader(0), 6, pre_hooks=[_Poison(3)], checkpointer=ck)
    steps = sorted(step for step, _, _ in scan_checkpoint_root(str(tmp_path)))
    assert steps and max(steps) == 3  # steps 1..3 saved; the NaN step (it would be step 4) never is
    assert tr.step == 4  # the step ran, the loop stopped on reading its loss


def _dp_rank(rank, world, root, phase):
    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.train.checkpoint import load_checkpoint, save_checkpoint

    ctx = pdist.init(ep_size=1, timeout_s=8 if phase == "fail" else 120)
    tr = _make(ctx)
    if phase == "fail":
        loader = _Loader(rank)
        for _ in range(2):
            tr.train_step(next(loader))
        save_checkpoint(tr, os.path.join(root, "step-2"))
        if rank == 1:
            return {"left": True}  # this rank leaves between steps: no kernel or collective in flight
        try:
            tr.train_step(next(loader))
        except Exception as e:  # the surviving rank's next collective fails within the short timeout
            return {"detected": type(e).__name__}
        return {"detected": None}
    if phase == "resume":
        load_checkpoint(tr, os.path.join(root, "step-2"))
        loader = _Loader(rank, start=tr.step)
    else:  # "straight": the unbroken reference run
        loader = _Loader(rank)
    while tr.step < 4:
        tr.train_step(next(loader))
    out = {"step": tr.step, "master": tr.store.master.numpy().copy()}  # numpy: safe to send after exit
    pdist.shutdown()
    return out


def test_rank_loss_is_detected_and_job_resumes(tmp_path):
    root = str(tmp_path)
    res = run_ranks(_dp_rank, 2, root, "fail", timeout=240)
    assert res[1] == {"left": True}
    assert res[0]["detected"] is not None, "the surviving rank did not notice the missing peer"
    assert os.path.exists(os.path.join(root, "step-2", "metadata.json"))
    resumed = run_ranks(_dp_rank, 2, root, "resume", timeout=240)
    straight = run_ranks(_dp_rank, 2, root, "straight", timeout=240)
    for r in range(2):
        assert resumed[r]["step"] == straight[r]["step"] == 4
        assert (resumed[r]["master"] == straight[r]["master"]).all()
