"""Evaluation: mean next-token loss (and bits per byte) of the current and EMA weights over held-out
batches (levanter's tagged evaluator as configured by ``GrugEvalConfig``,
megagpt-speedrun/train.py:175-222 and megagpt-speedrun/launch.py:170-190).

``bytes_per_token`` converts nats/token into bits/byte (``loss / ln 2 / bytes_per_token``); it is
1.0 for the byte tokenizer and measured from the corpus for others.
"""

from __future__ import annotations

import math

import torch


@torch.no_grad()
def evaluate(trainer, batches, *, prefix: str = "eval", bytes_per_token: float | None = None,
             max_batches: int | None = None, model_kwargs: dict | None = None) -> dict[str, float]:
    tot = torch.zeros((), dtype=torch.float64, device=trainer.device)
    n = 0
    for i, b in enumerate(batches):
        if max_batches is not None and i >= max_batches:
            break
        tok = b["tokens"].to(trainer.device, non_blocking=True)
        seg = b.get("segment_ids")
        seg = None if seg is None else seg.to(trainer.device, non_blocking=True)
        lw = b.get("loss_weight")
        lw = None if lw is None else lw.to(trainer.device, non_blocking=True)
        loss, met = trainer.model.next_token_loss(tok, lw, seg, z_loss_weight=0.0, dp_group=trainer.dp_group,
                                                  **(model_kwargs or {}))
        tot += met.get("train/cross_entropy_loss", loss).double()
        n += 1
    if trainer.dist is not None and trainer.dist.world > 1:
        import torch.distributed as tdist

        tdist.all_reduce(tot, group=trainer.dist.batch_group)
        tot /= trainer.dist.world
    loss = float(tot / max(n, 1))
    out = {f"{prefix}/loss": loss}
    if bytes_per_token:
        out[f"{prefix}/bpb"] = loss / math.log(2) / bytes_per_token
    return out


@torch.no_grad()
def evaluate_ema(trainer, batches, **kw) -> dict[str, float]:
    """Evaluate with the EMA weights swapped in, then restore the live weights."""
    if trainer.ema is None:
        return {}
    st = trainer.store
    live = st.master.clone()
    st.master.copy_(trainer.ema)
    st.sync_compute()
    try:
        return evaluate(trainer, batches, prefix=kw.pop("prefix", "eval") + "_ema", **kw)
    finally:
        st.master.copy_(live)
        st.sync_compute()


def evaluate_tagged(trainer, tagged: dict, *, prefix: str = "eval", max_batches: int | None = None,
                    model_kwargs: dict | None = None) -> dict[str, float]:
    """Loss per tag (domain) of ``tagged`` (tag -> batches), their unweighted mean (``macro_loss``)
    and the mean weighted by each tag's batch count (``micro_loss``), the breakdown of the
    reference's tagged evaluator (reentrant/eval_sweep.py:116-135)."""
    out: dict[str, float] = {}
    losses, counts = [], []
    for tag, batches in tagged.items():
        bl = list(batches)[:max_batches] if max_batches is not None else list(batches)
        r = evaluate(trainer, bl, prefix=f"{prefix}/{tag}", model_kwargs=model_kwargs)
        out.update(r)
        losses.append(r[f"{prefix}/{tag}/loss"])
        counts.append(len(bl))
    if losses:
        out[f"{prefix}/macro_loss"] = sum(losses) / len(losses)
        out[f"{prefix}/micro_loss"] = sum(l * c for l, c in zip(losses, counts)) / max(sum(counts), 1)
    return out


@torch.no_grad()
def evaluate_at_depths(trainer, batches, depths, *, prefix: str = "eval", max_batches: int | None = None
                       ) -> dict[int, dict[str, float]]:
    """A weight-tied looped model evaluated at several recurrence depths R: the same batches (a
    list, or tag -> list for the tagged breakdown) with the core looped R times. Returns
    R -> metrics (prefixed ``<prefix>/R<R>``) (reentrant/eval_sweep.py:99-135)."""
    res = {}
    for r in depths:
        kw = {"recurrence": int(r)}
        if isinstance(batches, dict):
            res[r] = evaluate_tagged(trainer, batches, prefix=f"{prefix}/R{r}", max_batches=max_batches, model_kwargs=kw)
        else:
            res[r] = evaluate(trainer, batches, prefix=f"{prefix}/R{r}", max_batches=max_batches, model_kwargs=kw)
    return res
