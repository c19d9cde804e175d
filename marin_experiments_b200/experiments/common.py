"""Launch config shared by the experiment launchers (the fields of the reference's
``GrugMoeLaunchConfig`` / ``TinyStoriesLaunchConfig``, megagpt-speedrun/launch.py:83-126,
tiny-stories/launch.py:96-113) and ``run_inline``, which turns one into a ``GrugRunConfig`` and
trains in-process (megagpt-speedrun/launch.py:128-198)."""

from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field

from ..config import (CheckpointerConfig, DataConfig, GrugEvalConfig, GrugModelConfig, GrugRunConfig,
                      GrugTrainerConfig, TrainerConfig)


def temporary_checkpoint_base_path(output_path: str) -> str:
    return os.path.join(output_path, "checkpoints-temp")


@dataclass(frozen=True)
class GrugLaunchConfig:
    model: GrugModelConfig
    data: DataConfig
    output_path: str
    run_id: str
    steps: int
    batch_size: int
    seed: int = 0
    mp: str = "params=float32,compute=bfloat16,output=bfloat16"
    optimizer: object = None
    grug_trainer: GrugTrainerConfig = field(default_factory=GrugTrainerConfig)
    eval: GrugEvalConfig | None = None
    checkpointer: CheckpointerConfig | None = None
    tracker: str = field(default_factory=lambda: os.environ.get("MXK_TRACKER", "jsonl"))  # jsonl | wandb | noop
    k_schedule: tuple | None = None
    init_from: str | None = None
    per_device_parallelism: int = -1
    save_interval_s: float = 30 * 60
    keep: tuple | None = None
    eval_only: bool = False
    # a models.looped.LoopedConfig: train the re-entrant (looped) variant of ``model`` instead
    looped: object = None


def to_run_config(c: GrugLaunchConfig) -> GrugRunConfig:
    ck = c.checkpointer or CheckpointerConfig(
        base_path=os.path.join(c.output_path, "checkpoints"),
        temporary_base_path=temporary_checkpoint_base_path(c.output_path), append_run_id_to_base_path=False,
        save_interval_s=c.save_interval_s, keep_last_temporary_checkpoints=2, keep=c.keep)
    trainer = TrainerConfig(id=c.run_id, seed=c.seed, num_train_steps=c.steps, train_batch_size=c.batch_size,
                            per_device_parallelism=c.per_device_parallelism, mp=c.mp, checkpointer=ck,
                            initialize_from=c.init_from)
    return GrugRunConfig(model=c.model, data=dataclasses.replace(c.data, seq_len=c.model.max_seq_len),
                         optimizer=c.optimizer, trainer=dataclasses.replace(c.grug_trainer, trainer=trainer),
                         eval=c.eval, k_schedule=c.k_schedule, output_path=c.output_path)


def run_inline(c: GrugLaunchConfig) -> dict:
    from ..train.run import run_grug

    factory = None
    if c.looped is not None:
        from ..models.looped import LoopedTransformer

        lc = dataclasses.replace(c.looped, model=c.model)
        factory = lambda cfg, local: LoopedTransformer(dataclasses.replace(lc, model=cfg))  # noqa: E731
    return run_grug(to_run_config(c), tracker=c.tracker, eval_only=c.eval_only, model_factory=factory)
