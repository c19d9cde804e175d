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
             max_batches: int | None = None) -> dict[str, float]:
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
        loss, met = trainer.model.next_token_loss(tok, lw, seg, z_loss_weight=0.0, dp_group=trainer.dp_group)
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
