"""Re-entrant (looped) grug MoE: prelude -> shared core applied R times -> coda
(reentrant/model.py:82-237,686-965; R sampled per step in reentrant/train.py:516-522).

Knobs (all off by default, so a ``LoopedConfig`` with R = 1 is the plain grug stack):

* ``recurrence_steps`` R: the weight-tied core (layers between prelude and coda) runs R times;
  ``randomize_recurrence`` draws R per training step from ``recurrence_choices``.
* ``iteration_film``: per (iteration, core layer) learned feature scale/shift applied to the core
  block's input, ``x * (1 + s) + b``; zero-initialised, so step 0 equals the untied stack.
* ``depth_conditioned_routing``: per (iteration, core layer) learned additive router-logit bias (a
  real part of the logits, with gradient), zero-initialised.
* ``core_consistency_weight``: penalty on the normalised squared change of the hidden state between
  consecutive core iterations.
* ``anytime_supervision``: extra CE read off the shared head after every core iteration, averaged
  over iterations.
* ``ponder_halting``: PonderNet -- a halting head on each iteration's readout gives a halting
  distribution; adds the expected CE under it plus ``KL(halting || geometric prior)``.

Iterations beyond the largest trained depth reuse the last FiLM / routing-bias entry (test-time depth
scaling).
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field

import torch
from torch import nn

from ..config import GrugModelConfig
from ..ops import api as ops
from .grug import Transformer, combine_losses, default_loss_weight


@dataclass(frozen=True)
class LoopedConfig:
    model: GrugModelConfig = field(default_factory=GrugModelConfig)
    num_prelude_layers: int = 0
    num_coda_layers: int = 0
    recurrence_steps: int = 1
    iteration_film: bool = False
    randomize_recurrence: bool = False
    recurrence_choices: tuple[int, ...] = ()
    core_consistency_weight: float = 0.0
    depth_conditioned_routing: bool = False
    anytime_supervision: bool = False
    anytime_supervision_weight: float = 1.0
    ponder_halting: bool = False
    ponder_loss_weight: float = 1.0
    ponder_kl_weight: float = 0.01
    ponder_prior_lambda: float = 0.2

    def __post_init__(self):
        m = self.model
        if self.num_prelude_layers < 0 or self.num_coda_layers < 0:
            raise ValueError("num_prelude_layers and num_coda_layers must be non-negative")
        if self.num_prelude_layers + self.num_coda_layers > m.num_layers:
            raise ValueError("num_prelude_layers + num_coda_layers must be <= num_layers")
        if self.recurrence_steps < 1:
            raise ValueError("recurrence_steps must be >= 1")
        if self.recurrence_steps > 1 and self.num_core_layers <= 0:
            raise ValueError("recurrence_steps > 1 requires at least one core layer")
        if self.randomize_recurrence:
            if not self.recurrence_choices:
                raise ValueError("randomize_recurrence requires a non-empty recurrence_choices")
            if any(c < 1 for c in self.recurrence_choices):
                raise ValueError("recurrence_choices must all be >= 1")

    @property
    def num_core_layers(self) -> int:
        return self.model.num_layers - self.num_prelude_layers - self.num_coda_layers

    @property
    def table_depth(self) -> int:
        return max([self.recurrence_steps, *self.recurrence_choices])

    def effective_depth(self, r: int | None = None) -> int:
        r = self.recurrence_steps if r is None else r
        return self.num_prelude_layers + self.num_core_layers * r + self.num_coda_layers


class LoopedTransformer(nn.Module):
    def __init__(self, lc: LoopedConfig):
        super().__init__()
        self.lc = lc
        self.cfg = lc.model
        self.base = Transformer(lc.model)
        d, c, td = lc.model.hidden_dim, lc.num_core_layers, lc.table_depth
        self.film_scale = nn.Parameter(torch.zeros(td, c, d)) if lc.iteration_film else None
        self.film_shift = nn.Parameter(torch.zeros(td, c, d)) if lc.iteration_film else None
        self.depth_bias = (nn.Parameter(torch.zeros(td, c, lc.model.num_experts))
                           if lc.depth_conditioned_routing and lc.model.is_moe else None)
        self.halt_head = nn.Parameter(torch.zeros(d)) if lc.ponder_halting else None

    @property
    def blocks(self):
        """The unique layers (prelude, core, coda): what QB router biases are kept for."""
        return self.base.blocks

    @property
    def prelude(self):
        return self.base.blocks[: self.lc.num_prelude_layers]

    @property
    def core(self):
        p = self.lc.num_prelude_layers
        return self.base.blocks[p: p + self.lc.num_core_layers]

    @property
    def coda(self):
        return self.base.blocks[self.lc.num_prelude_layers + self.lc.num_core_layers:]

    def init_weights(self, seed: int = 0):
        self.base.init_weights(seed)
        for p in (self.film_scale, self.film_shift, self.depth_bias, self.halt_head):
            if p is not None:
                p.data.zero_()
        return self

    def sample_recurrence(self, rng: random.Random) -> int:
        if self.lc.randomize_recurrence:
            return rng.choice(self.lc.recurrence_choices)
        return self.lc.recurrence_steps

    def forward(self, tokens, segment_ids=None, dp_group=None, recurrence: int | None = None):
        """Returns ``(h_final, stats, readouts, consistency)``."""
        lc = self.lc
        b, s = tokens.shape
        seg = None if segment_ids is None else segment_ids.reshape(-1)
        x = self.base.embed(tokens)
        stats = []
        for blk in self.prelude:
            x, st = blk(x, b, s, seg, dp_group)
            stats += [st] if st is not None else []
        r = lc.recurrence_steps if recurrence is None else recurrence
        readouts, cons, prev = [], None, None
        for it in range(r):
            ti = min(it, lc.table_depth - 1)
            for li, blk in enumerate(self.core):
                if self.film_scale is not None:
                    x = x * (1 + self.film_scale[ti, li].to(x.dtype)) + self.film_shift[ti, li].to(x.dtype)
                lb = self.depth_bias[ti, li] if self.depth_bias is not None else None
                x, st = blk(x, b, s, seg, dp_group, logit_bias=lb)
                stats += [st] if st is not None else []
            if lc.core_consistency_weight and prev is not None:
                pf, xf = prev.float(), x.float()
                term = (xf - pf).pow(2).mean() / pf.pow(2).mean().clamp_min(1e-6)
                cons = term if cons is None else cons + term
            if lc.core_consistency_weight:
                prev = x
            if lc.anytime_supervision or lc.ponder_halting:
                readouts.append(x)
        for blk in self.coda:
            x, st = blk(x, b, s, seg, dp_group)
            stats += [st] if st is not None else []
        if cons is not None and r > 1:
            cons = cons / (r - 1)
        return self.base.head_input(x), stats, readouts, cons

    # ------------------------------------------------------------------------------- loss
    def next_token_loss(self, tokens, loss_weight=None, segment_ids=None, *, z_loss_weight: float = 0.0,
                        dp_group=None, recurrence: int | None = None):
        lc = self.lc
        b, s = tokens.shape
        h, stats, readouts, cons = self.forward(tokens, segment_ids, dp_group, recurrence)
        labels = torch.cat([tokens[:, 1:], torch.zeros_like(tokens[:, :1])], dim=1).reshape(-1)
        if loss_weight is None:
            loss_weight = default_loss_weight(b, s, tokens.device)
        w = loss_weight.reshape(-1).float()
        ce = ops.cross_entropy(h, self.base.head_weight(), labels, w, z_weight=z_loss_weight)
        loss, metrics = combine_losses(self.cfg, ce, stats)
        if "qb_beta_per_layer" in metrics:  # one beta per unique layer: average a core layer's iterations
            bt = metrics["qb_beta_per_layer"]
            p, c = lc.num_prelude_layers, lc.num_core_layers
            r = (bt.shape[0] - p - lc.num_coda_layers) // max(c, 1)
            core = bt[p:p + r * c].reshape(r, c, -1).mean(0) if c else bt[p:p]
            metrics["qb_beta_per_layer"] = torch.cat([bt[:p], core, bt[p + r * c:]], 0)
        if cons is not None and lc.core_consistency_weight:
            loss = loss + lc.core_consistency_weight * cons
            metrics["train/core_consistency"] = cons.detach()
        if lc.anytime_supervision and readouts:
            terms = []
            wt = lc.anytime_supervision_weight / len(readouts)
            for rd in readouts:
                terms.append(self._weighted_ce(self.base.head_input(rd), labels, w, wt))
            any_ce = torch.stack([t for t, _ in terms]).sum()
            loss = loss + any_ce
            metrics["train/anytime_ce"] = torch.stack([v for _, v in terms]).mean()
        if lc.ponder_halting and readouts:
            pl, kl, halt = self._ponder(readouts, labels, w)
            loss = loss + lc.ponder_loss_weight * pl + lc.ponder_kl_weight * kl
            metrics.update({"train/ponder_ce": pl.detach(), "train/ponder_kl": kl.detach(),
                            "train/ponder_expected_steps": halt.detach()})
        metrics["train/loss"] = loss.detach()
        return loss, metrics

    def _weighted_ce(self, hr, labels, w, weight: float):
        """``weight * CE`` through the fused kernel: on CUDA the fused CE accumulates its weight
        gradient with the current loss-gradient scale, so the scale is multiplied by ``weight`` for
        this call."""
        if hr.is_cuda:
            from ..ops import cuda_fns

            base = cuda_fns._CE_GRAD_SCALE[0]
            cuda_fns.set_loss_grad_scale(base * weight)
            try:
                v = ops.cross_entropy(hr, self.base.head_weight(), labels, w)
            finally:
                cuda_fns.set_loss_grad_scale(base)
            return v * weight, v.detach()
        v = ops.cross_entropy(hr, self.base.head_weight(), labels, w)
        return v * weight, v.detach()

    def _ponder(self, readouts, labels, w, chunk: int = 4096):
        """PonderNet terms: halting probabilities from the halt head on each readout, the expected
        per-token CE under them, and KL to a truncated geometric prior."""
        lc = self.lc
        r = len(readouts)
        lam = [torch.sigmoid(self.base.head_input(rd).float() @ self.halt_head.float()) for rd in readouts]
        probs, surv = [], torch.ones_like(lam[0])
        for i in range(r):
            p = surv * lam[i] if i < r - 1 else surv
            probs.append(p)
            surv = surv * (1 - lam[i])
        P = torch.stack(probs, 0)  # [R, T]
        W = self.base.head_weight().float()
        ces = []
        for rd in readouts:
            hr = self.base.head_input(rd).float()
            parts = []
            for t0 in range(0, hr.shape[0], chunk):
                lg = hr[t0:t0 + chunk] @ W.t()
                parts.append(torch.logsumexp(lg, -1) - lg.gather(1, labels[t0:t0 + chunk, None]).squeeze(1))
            ces.append(torch.cat(parts))
        C = torch.stack(ces, 0)  # [R, T]
        wsum = w.sum().clamp_min(1.0)
        expected = ((P * C).sum(0) * w).sum() / wsum
        lp = lc.ponder_prior_lambda
        prior = torch.tensor([lp * (1 - lp) ** i for i in range(r)], device=P.device)
        prior = prior / prior.sum()
        kl = ((P * (torch.log(P.clamp_min(1e-8)) - torch.log(prior)[:, None])).sum(0) * w).sum() / wsum
        steps = ((P * torch.arange(1, r + 1, device=P.device)[:, None]).sum(0) * w).sum() / wsum
        return expected, kl, steps
