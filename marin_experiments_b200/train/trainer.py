"""Training step and loop (megagpt-speedrun/train.py:420-775, tiny-stories/train.py:514-697).

``Trainer`` owns the model, its flat ``ParamStore``, the optimizer and the QB state. One
``train_step``:

1. copies the batch to the device (non-blocking from pinned memory),
2. sets every router bias from the previous step's QB betas, ``bias = -beta - mean(-beta)``
   (megagpt-speedrun/train.py:320-332),
3. optionally moves the weights to the forward predictor's point (delayed-gradient correctors),
4. runs ``n_micro`` forward/backward passes (gradients accumulate in fp32 ``main_grad``; each
   microbatch loss is scaled by ``1/n_micro``),
5. reduces gradients across data-parallel ranks (``grad_sync``),
6. applies the optimizer, the EMA, and stores the mean QB betas for the next step.

Returned metrics are device tensors; nothing in the step synchronises with the host unless a
caller reads them.
"""

from __future__ import annotations

import math
import time

import torch

from ..config import GrugModelConfig, GrugRunConfig
from ..models.grug import MoEMLP, Transformer, apply_qb_betas, default_loss_weight, init_store_weights
from ..utils.profiling import nvtx_range, watch_stats
from .params import ParamStore


def num_moe_layers(model: Transformer) -> int:
    return sum(1 for b in model.blocks if isinstance(b.mlp, MoEMLP))


class Trainer:
    def __init__(self, cfg: GrugRunConfig, *, device: str | torch.device | None = None, micro_batch: int | None = None,
                 num_train_steps: int | None = None, dist=None, build_model: bool = True, seed: int | None = None,
                 model_kwargs: dict | None = None, model_factory=None):
        self.cfg = cfg
        self.mcfg: GrugModelConfig = cfg.model
        if device is None:
            device = "cuda" if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        self.dist = dist
        self.step = 0
        self.num_train_steps = num_train_steps or cfg.trainer.trainer.num_train_steps
        self.micro_batch = micro_batch
        self.seed = cfg.trainer.trainer.seed if seed is None else seed
        self.z_loss_weight = cfg.trainer.z_loss_weight
        self.ema_beta = cfg.trainer.ema_beta
        self.model_kwargs = dict(model_kwargs or {})
        # model_factory(cfg, local_experts) -> module with next_token_loss (e.g. the looped model)
        self.model_factory = model_factory
        import random as _random

        self._rng = _random.Random(self.seed)
        if build_model:
            self._build()

    # ------------------------------------------------------------------------------- build
    def _build(self) -> None:
        cfg = self.mcfg
        local = None
        if self.dist is not None and self.dist.ep_size > 1 and cfg.is_moe:
            local = self.dist.local_expert_range(cfg.num_experts)
        with torch.device("meta"):
            if self.model_factory is not None:
                model = self.model_factory(cfg, local)
            else:
                model = Transformer(cfg, local_experts=local, **self.model_kwargs)
        self.model = model
        self.store = ParamStore(model, self.device, pad_multiple=getattr(self.dist, "store_pad", 64),
                                expert_last=getattr(self.dist, "expert_last", False),
                                alloc=getattr(self.dist, "store_alloc", None))
        init_store_weights(self.store, cfg, self.seed, model)
        if self.dist is not None:
            self.dist.setup_model(self)
        opt_cfg = self.cfg.optimizer
        if opt_cfg is None:
            from ..optim import GrugMoeAdamHConfig

            opt_cfg = GrugMoeAdamHConfig()
        self.opt = opt_cfg.build(self.store, self.num_train_steps)
        if self.dist is not None:
            self.dist.setup_optimizer(self)
        n_moe = num_moe_layers(model)
        self.pending_qb = torch.zeros(max(n_moe, 1), max(cfg.num_experts, 1), device=self.device) if n_moe else None
        self.ema = self.store.master.clone() if self.ema_beta is not None else None
        self.watch_every, self.watch_per_param, self.watch_hist_bins = 0, False, 0  # set by run_grug

    @property
    def dp_group(self):
        return None if self.dist is None else self.dist.batch_group

    # ------------------------------------------------------------------------------- step
    def _to_device(self, t: torch.Tensor | None):
        if t is None:
            return None
        return t.to(self.device, non_blocking=True)

    def train_step(self, batch: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        from ..ops import cuda_fns  # noqa: F401 (loss-scale contract of the fused CE)

        tokens = self._to_device(batch["tokens"])
        seg = self._to_device(batch.get("segment_ids"))
        lw = self._to_device(batch.get("loss_weight"))
        b, s = tokens.shape
        mb = self.micro_batch or b
        if b % mb:
            raise ValueError(f"local batch {b} is not a multiple of the microbatch {mb}")
        n_micro = b // mb
        if self.pending_qb is not None and self.mcfg.qb_balancing:
            apply_qb_betas(self.model, self.pending_qb)
        predictor = getattr(self.opt, "has_forward_predictor", None)
        use_pred = predictor is not None and self.opt.has_forward_predictor()
        if use_pred:
            self.opt.apply_forward_offset()
        if self.device.type == "cuda":
            cuda_fns.set_loss_grad_scale(1.0 / n_micro)
        loss_sum = torch.zeros((), device=self.device)
        beta_sum = None
        metrics: dict[str, torch.Tensor] = {}
        extra = {}
        if hasattr(self.model, "sample_recurrence"):  # looped model: depth drawn once per step
            extra["recurrence"] = self.model.sample_recurrence(self._rng)
        for i in range(n_micro):
            sl = slice(i * mb, (i + 1) * mb)
            if i == n_micro - 1 and self.dist is not None and hasattr(self.dist, "arm_overlap"):
                self.dist.arm_overlap()  # the last backward starts the gradient reductions
            w = lw[sl] if lw is not None else default_loss_weight(mb, s, self.device)
            with nvtx_range(f"microbatch{i}"):
                loss, met = self.model.next_token_loss(tokens[sl], w, None if seg is None else seg[sl],
                                                       z_loss_weight=self.z_loss_weight, dp_group=self.dp_group,
                                                       **extra)
                (loss / n_micro).backward()
            loss_sum = loss_sum + loss.detach()
            if "qb_beta_per_layer" in met:
                beta_sum = met["qb_beta_per_layer"] if beta_sum is None else beta_sum + met["qb_beta_per_layer"]
            for k, v in met.items():
                if k == "qb_beta_per_layer":
                    continue
                metrics[k] = v if k not in metrics else metrics[k] + v
        for k in list(metrics):
            if k != "routing_counts_per_layer":
                metrics[k] = metrics[k] / n_micro
        if use_pred:
            self.opt.restore_weights()
        if self.dist is not None:
            with nvtx_range("grad_sync"):
                self.dist.grad_sync(self)
        if self.watch_every and self.step % self.watch_every == 0:
            metrics.update(watch_stats(self.store, per_param=self.watch_per_param, hist_bins=self.watch_hist_bins,
                                       ep_group=getattr(self.dist, "ep_group", None) if self.dist else None))
        with nvtx_range("optimizer"):
            self.opt.step()
        if self.dist is not None and hasattr(self.dist, "post_step"):
            self.dist.post_step(self)
        if beta_sum is not None:
            self.pending_qb = beta_sum / n_micro
        if self.ema is not None:
            self.ema.mul_(self.ema_beta).add_(self.store.master, alpha=1 - self.ema_beta)
        self.step += 1
        metrics["train/loss"] = loss_sum / n_micro
        return metrics

    # ------------------------------------------------------------------------------ loop
    def fit(self, loader, num_steps: int, *, hooks=(), pre_hooks=(), log_every: int = 1, checkpointer=None,
            tracker=None, stop_on_nan: bool = True):
        """Hot loop: batch -> step -> host read of the loss -> NaN stop -> hooks/tracker ->
        checkpoint (megagpt-speedrun/train.py:705-762)."""
        it = iter(loader)
        last = None
        while self.step < num_steps:
            for h in pre_hooks:
                h.before_step(self)
            t0 = time.perf_counter()
            batch = next(it)
            t_load = time.perf_counter() - t0
            met = self.train_step(batch)
            loss = float(met["train/loss"].item())
            dt = time.perf_counter() - t0
            if stop_on_nan and not math.isfinite(loss):
                raise FloatingPointError(f"loss is {loss} at step {self.step}")
            info = {"step": self.step, "loss": loss, "step_duration": dt, "loading_time": t_load,
                    "tokens": int(batch["tokens"].numel()) * (self.dist.world if self.dist else 1),
                    "batch_size": int(batch["tokens"].shape[0]) * (self.dist.world if self.dist else 1),
                    "metrics": met}
            t_h = time.perf_counter()
            for h in hooks:
                h(self, info)
            hook_time = time.perf_counter() - t_h
            if tracker is not None and self.step % log_every == 0:
                from ..utils.tracker import router_layer_metrics

                perf = {"throughput/step_duration": dt, "throughput/loading_time": t_load,
                        "throughput/hook_time": hook_time}
                for h in hooks:  # e.g. the throughput hook's tokens/s and MFU of this step
                    last_h = getattr(h, "last", None)
                    if isinstance(last_h, dict):
                        perf.update(last_h)
                tracker.log({**{k: (float(v.float().mean()) if torch.is_tensor(v) else v) for k, v in met.items()
                                if not (torch.is_tensor(v) and v.numel() > 1)}, **router_layer_metrics(met),
                             **perf}, step=self.step)
            if checkpointer is not None:
                checkpointer.on_step(self, self.step)
            last = info
        if checkpointer is not None:
            checkpointer.on_step(self, self.step, force=True)
        return last
