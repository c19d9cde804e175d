"""Training entry: ``run_grug(GrugRunConfig)`` (megagpt-speedrun/train.py:513-775).

Wires the pieces of a run: process group and expert-parallel mesh (one process per GPU), the
trainer, the native data loader, checkpoint restore (newest-first with fallback) or a weights-only
``initialize_from`` graft, the k-curriculum, eval-only mode, throughput logging, the step watchdog,
the hot loop with its NaN stop, and the final checkpoint.
"""

from __future__ import annotations

import os

import torch

from ..config import GrugRunConfig, to_dict
from ..data.loader import DataLoader, build_dataset
from ..utils.profiling import ProfilerHook
from ..utils.tracker import ThroughputHook, Watchdog, make_tracker
from .checkpoint import Checkpointer, initialize_from, restore_from_checkpoint
from .curriculum import KCurriculumHook
from .eval import evaluate, evaluate_ema
from .trainer import Trainer


def _device() -> torch.device:
    """``ACCELERATOR`` (``cpu`` / ``gpu``, the launchers' switch of tiny-stories/launch.py:55-84)
    picks the device; unset, a GPU is used when there is one."""
    acc = os.environ.get("ACCELERATOR", "").lower()
    if acc not in ("", "cpu", "gpu"):
        raise ValueError(f"ACCELERATOR={acc!r}: this framework runs on cpu or gpu")
    if acc == "gpu" and not torch.cuda.is_available():
        raise RuntimeError("ACCELERATOR=gpu but no CUDA device is visible")
    if acc != "cpu" and torch.cuda.is_available():
        idx = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(idx)
        return torch.device("cuda", idx)
    return torch.device("cpu")


def run_grug(cfg: GrugRunConfig, *, tracker: str = "jsonl", hooks=(), eval_only: bool = False,
             device: torch.device | None = None, peak_flops_per_gpu: float = 2.25e15, model_factory=None) -> dict:
    tcfg = cfg.trainer.trainer
    dist_ctx = None
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        from ..parallel import dist as pdist

        dist_ctx = pdist.init(ep_size=cfg.trainer.expert_axis_size)
    device = device or _device()
    rank = dist_ctx.rank if dist_ctx else 0
    world = dist_ctx.world if dist_ctx else 1
    run_id = tcfg.id or "grug"
    micro = tcfg.per_device_parallelism if tcfg.per_device_parallelism > 0 else None
    trainer = Trainer(cfg, device=device, micro_batch=micro, num_train_steps=tcfg.num_train_steps, dist=dist_ctx,
                      model_factory=model_factory)
    ck_cfg = tcfg.checkpointer
    if not os.path.isabs(ck_cfg.base_path):
        import dataclasses

        tmp = ck_cfg.temporary_base_path
        ck_cfg = dataclasses.replace(
            ck_cfg, base_path=os.path.join(cfg.output_path, ck_cfg.base_path),
            temporary_base_path=None if tmp is None else (tmp if os.path.isabs(tmp) else os.path.join(cfg.output_path, tmp)))
    ckpt = Checkpointer(ck_cfg, run_id=run_id)
    search = [tcfg.load_checkpoint_path] if tcfg.load_checkpoint_path else ckpt.search_paths()
    restored = restore_from_checkpoint(trainer, search, allow_partial=tcfg.allow_partial_checkpoint)
    if restored is None and tcfg.initialize_from:
        initialize_from(trainer, tcfg.initialize_from)
    trk = make_tracker(tracker, os.path.join(cfg.output_path, tcfg.log_dir), run_id, to_dict(cfg), rank)
    seq = cfg.model.max_seq_len
    ds = build_dataset(cfg.data, seq, cfg.model.vocab_size)
    result: dict = {"restored_from": restored, "start_step": trainer.step}

    ev = cfg.eval
    eval_batches = None
    if ev is not None:
        import dataclasses

        eds = build_dataset(dataclasses.replace(cfg.data, seed=cfg.data.seed + 7919), seq, cfg.model.vocab_size)
        eb = max(world, min(ev.eval_batch_size, tcfg.train_batch_size))
        n_eval = ev.max_eval_batches or 4

        def eval_batches():
            dl = DataLoader(eds, eb, rank=rank, world=world, depth=2)
            return (next(dl) for _ in range(n_eval))

    def run_eval(step: int) -> dict:
        out = {}
        if ev.eval_current:
            out.update(evaluate(trainer, eval_batches(), prefix=ev.prefix))
        if ev.eval_ema and trainer.ema is not None:
            out.update(evaluate_ema(trainer, eval_batches(), prefix=ev.prefix))
        trk.log(out, step=step)
        return out

    if eval_only:
        result["eval"] = run_eval(trainer.step) if ev is not None else {}
        trk.finish()
        return result

    loader = DataLoader(ds, tcfg.train_batch_size, rank=rank, world=world, start_step=trainer.step)
    thr = ThroughputHook(cfg.model, world, peak_flops_per_gpu, every=cfg.trainer.log_every)
    wd = Watchdog(tcfg.watchdog_timeout_s).start()
    trainer.watch_every, trainer.watch_per_param = tcfg.watch_every, tcfg.watch_per_param
    trainer.watch_hist_bins = tcfg.watch_hist_bins
    all_hooks = [thr, wd, *hooks]
    pre = [KCurriculumHook(cfg.k_schedule)] if cfg.k_schedule else []
    if tcfg.profiler:
        prof = ProfilerHook(os.path.join(cfg.output_path, tcfg.log_dir, run_id, "profiler"), tcfg.profiler_start_step,
                            tcfg.profiler_num_steps, rank)
        pre.append(prof)
        all_hooks.append(prof)
    if ev is not None and ev.steps_per_eval:
        def eval_hook(tr, info):
            if info["step"] % ev.steps_per_eval == 0:
                info["eval"] = run_eval(info["step"])
        all_hooks.append(eval_hook)
    try:
        last = trainer.fit(loader, tcfg.num_train_steps, hooks=all_hooks, pre_hooks=pre,
                           log_every=cfg.trainer.log_every, tracker=trk, checkpointer=ckpt)
    finally:
        wd.stop()
    ckpt.on_end(trainer)
    trk.log_summary({"final_step": trainer.step, **({} if last is None else {"final_loss": last["loss"]})})
    trk.finish()
    result.update(final_step=trainer.step, final_loss=None if last is None else last["loss"], trainer=trainer,
                  checkpointer=ckpt)
    return result
