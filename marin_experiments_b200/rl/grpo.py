"""GRPO and Dr.GRPO objectives (tunix-delphi-rl/training/train_coding.py:14-40 describes the Dr.GRPO
variant the reference trains with).

For a group of G completions of one prompt with rewards ``r``:

* GRPO advantage ``(r - mean(r)) / (std(r) + eps)``, loss averaged per response over its tokens;
* Dr.GRPO advantage ``r - mean(r)`` (no std division), loss summed over tokens and divided by a
  constant (``G * max_len``), so long responses are not down-weighted per token.

The token loss is the clipped importance-weighted policy gradient
``-min(rho A, clip(rho, 1-eps, 1+eps) A)`` with ``rho = exp(logp - logp_old)`` (``rho = 1`` on the
first pass when ``logp_old`` is the detached ``logp``), plus ``beta * KL(pi || pi_ref)`` (k3 estimator)
when reference log-probs are given.
"""

from __future__ import annotations

import torch


def group_advantages(rewards: torch.Tensor, group_size: int, variant: str = "dr_grpo", eps: float = 1e-6):
    r = rewards.view(-1, group_size).float()
    a = r - r.mean(1, keepdim=True)
    if variant == "grpo":
        a = a / (r.std(1, keepdim=True, unbiased=False) + eps)
    elif variant != "dr_grpo":
        raise ValueError(f"unknown variant {variant}")
    return a.reshape(-1)


def policy_loss(logp: torch.Tensor, mask: torch.Tensor, adv: torch.Tensor, *, logp_old: torch.Tensor | None = None,
                logp_ref: torch.Tensor | None = None, clip_eps: float = 0.2, beta: float = 0.0,
                variant: str = "dr_grpo", max_len: int | None = None):
    """``logp``, ``mask`` ``[N, L]`` (completion tokens), ``adv`` ``[N]``. Returns (loss, metrics)."""
    old = logp.detach() if logp_old is None else logp_old
    rho = torch.exp(logp - old)
    a = adv[:, None]
    tok = -torch.minimum(rho * a, rho.clamp(1 - clip_eps, 1 + clip_eps) * a)
    kl = None
    if logp_ref is not None and beta > 0:
        d = logp_ref - logp
        kl = torch.exp(d) - d - 1
        tok = tok + beta * kl
    m = mask.float()
    if variant == "dr_grpo":
        denom = float(mask.shape[0] * (max_len or mask.shape[1]))
        loss = (tok * m).sum() / denom
    else:
        loss = ((tok * m).sum(1) / m.sum(1).clamp_min(1)).mean()
    met = {"clip_frac": (((rho - 1).abs() > clip_eps).float() * m).sum() / m.sum().clamp_min(1)}
    if kl is not None:
        met["kl"] = (kl * m).sum() / m.sum().clamp_min(1)
    return loss, met


def sequence_logprobs(logits: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    """Per-token log-probabilities of ``tokens[:, 1:]`` under ``logits[:, :-1]``."""
    lp = torch.log_softmax(logits[:, :-1].float(), -1)
    return lp.gather(-1, tokens[:, 1:, None]).squeeze(-1)
