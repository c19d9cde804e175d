"""Delayed-gradient optimizer wrapper (pipeline-parallel staleness), on flat buffers.

Behaviour follows delayed-gradient-pp/delay_optim.py:78-416:

* every parameter's gradient is delayed by its own tau (uniform ``tau``, or the per-stage profile
  ``grug_stage_tau`` where the last pipeline stage is fresh and the embeddings are stalest);
  ``tau == 0`` is a pass-through, bit-identical to the inner optimizer;
* correctors applied to the stale gradient: ``none``, ``dc_asgd`` (g + lambda g*g (w_t - w_stale)),
  ``dc_asgd_ema`` (curvature from an EMA of g^2), ``lr_damp`` (scales the applied update);
* forward predictors (the train step evaluates the gradient at ``w + offset``): ``weight_pred``
  (offset = tau * pred_scale * last applied update) and the raw-momentum family ``wp_preorth``,
  ``wp_cautious``, ``wp_trust``, ``wp_confidence``.

The gradient history is a ring buffer ``[tau_max, N]`` over the store's flat gradient layout.
"""

from __future__ import annotations

import re
from dataclasses import dataclass

import torch

from .base import register
from .configs import GrugMoeAdamHConfig, MuonConfig

CORRECTORS = ("none", "dc_asgd", "dc_asgd_ema", "weight_pred", "lr_damp", "wp_preorth", "wp_cautious",
              "wp_trust", "wp_confidence")
FORWARD_PRED = ("weight_pred", "wp_preorth", "wp_cautious", "wp_trust", "wp_confidence")
PREORTH = ("wp_preorth", "wp_cautious", "wp_trust", "wp_confidence")
INPUT_FIELDS = ("token_embed", "embed_norm", "embed_up")
OUTPUT_FIELDS = ("output_proj", "final_norm", "head_down")
EPS = 1e-12


def grug_stage_tau(num_layers: int, num_stages: int):
    """Per-parameter delay of a ``num_stages``-stage pipeline over ``num_layers`` blocks: block i is
    in stage ``i * P // L`` with delay ``P - 1 - stage``; input-side parameters get ``P - 1``,
    output-side ones 0 (delayed-gradient-pp/delay_optim.py:103-128)."""
    if num_stages < 1 or num_layers < 1:
        raise ValueError(f"num_layers and num_stages must be >= 1, got {num_layers}, {num_stages}")

    def leaf_tau(name: str) -> int:
        m = re.search(r"blocks\.(\d+)\.", name)
        if m:
            stage = (int(m.group(1)) * num_stages) // num_layers
            return (num_stages - 1) - stage
        if any(f in name for f in INPUT_FIELDS):
            return num_stages - 1
        return 0

    return leaf_tau


def _rms(x: torch.Tensor) -> torch.Tensor:
    return torch.sqrt((x.float() ** 2).mean() + EPS)


class DelayedOptimizer:
    def __init__(self, inner, store, *, tau: int, corrector: str = "none", dc_lambda: float = 1.0,
                 dc_beta2: float = 0.99, lr_damp: float = 1.0, pred_beta: float = 0.95, pred_scale: float = 1.0,
                 trust: float = 0.01, leaf_tau=None):
        if tau < 0:
            raise ValueError(f"tau must be non-negative, got {tau}")
        if corrector not in CORRECTORS:
            raise ValueError(f"unknown corrector {corrector!r}; expected one of {CORRECTORS}")
        self.inner, self.store = inner, store
        self.corrector, self.dc_lambda, self.dc_beta2 = corrector, dc_lambda, dc_beta2
        self.damp = lr_damp if corrector == "lr_damp" else 1.0
        self.pred_beta, self.pred_scale, self.trust = pred_beta, pred_scale, trust
        self.taus = {i.name: (tau if leaf_tau is None else int(leaf_tau(i.name))) for i in store.infos}
        self.tau_max = max(self.taus.values()) if self.taus else 0
        n, dev = store.numel, store.device
        self.grad_ring = torch.zeros(self.tau_max, n, device=dev) if self.tau_max else None
        self.needs_w = corrector in ("dc_asgd", "dc_asgd_ema")
        self.param_ring = store.master.detach().clone().unsqueeze(0).repeat(self.tau_max, 1) \
            if (self.needs_w and self.tau_max) else None
        self.v_ema = torch.zeros(n, device=dev) if corrector == "dc_asgd_ema" else None
        self.m_raw = torch.zeros(n, device=dev) if corrector in PREORTH else None
        self.last_update = torch.zeros(n, device=dev)
        self.t = 0
        self._offset_backup = None

    # --------------------------------------------------------------------------- properties
    @property
    def step_count(self):
        return self.inner.step_count

    def current_lrs(self):
        return self.inner.current_lrs()

    def state_dict(self):
        sd = {"inner": self.inner.state_dict(), "t": self.t, "last_update": self.last_update.cpu()}
        if self.grad_ring is not None:
            sd["grad_ring"] = self.grad_ring.cpu()
        if self.param_ring is not None:
            sd["param_ring"] = self.param_ring.cpu()
        if self.v_ema is not None:
            sd["v_ema"] = self.v_ema.cpu()
        if self.m_raw is not None:
            sd["m_raw"] = self.m_raw.cpu()
        return sd

    def load_state_dict(self, sd):
        self.inner.load_state_dict(sd["inner"])
        self.t = int(sd["t"])
        self.last_update.copy_(sd["last_update"])
        for k in ("grad_ring", "param_ring", "v_ema", "m_raw"):
            if k in sd and getattr(self, k) is not None:
                getattr(self, k).copy_(sd[k])

    # -------------------------------------------------------------------------------- step
    def _delay_chunks(self):
        """(start, len, tau) chunks covering the whole flat buffer (alignment gaps with tau 0)."""
        import numpy as np

        if getattr(self, "_chunks", None) is None:
            rows, pos = [], 0
            for info in sorted(self.store.infos, key=lambda i: i.offset):
                if info.offset > pos:
                    rows.append((pos, info.offset - pos, 0))
                rows.append((info.offset, info.numel, self.taus[info.name]))
                pos = info.offset + info.numel
            if pos < self.store.numel:
                rows.append((pos, self.store.numel - pos, 0))
            out = []
            for s0, ln, tau in rows:
                for c0 in range(s0, s0 + ln, 32768):
                    out.append((c0, min(32768, s0 + ln - c0), tau))
            dt = np.dtype([("start", "<i8"), ("len", "<i4"), ("tau", "<i4")])
            arr = np.array(out, dtype=dt)
            self._chunks = torch.from_numpy(arr.view(np.uint8).copy()).to(self.store.device)
            self._nchunks = len(out)
        return self._chunks, self._nchunks

    @torch.no_grad()
    def _step_fused(self, grad_scale: float, zero_grad: bool) -> None:
        """The step as two sm_100a passes around the inner optimizer (``ops/csrc/delayed.cu``)."""
        from ..ops._ext import ext

        st = self.store
        chunks, nchunks = self._delay_chunks()
        cid = {"dc_asgd": 1, "dc_asgd_ema": 2}.get(self.corrector, 0)
        ext().delayed_prep(chunks, nchunks, st.grad, st.master, self.grad_ring, self.param_ring, self.v_ema,
                           self.m_raw, self.last_update, self.t, self.tau_max, cid, self.dc_lambda, self.dc_beta2,
                           self.pred_beta, grad_scale)
        self.inner.step(grad_scale=grad_scale, zero_grad=False)
        ext().delayed_finish(st.master, self.last_update, st.compute if self.damp != 1.0 else None, self.damp)
        self.t += 1
        if zero_grad:
            st.zero_grad()

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, zero_grad: bool = True) -> None:
        st = self.store
        if st.cuda:
            return self._step_fused(grad_scale, zero_grad)
        g_cur = st.grad.clone()
        if self.tau_max:
            for info in st.infos:
                tau = self.taus[info.name]
                if tau == 0:
                    continue
                sl = slice(info.offset, info.offset + info.numel)
                # the entry written tau steps ago (zeros while the FIFO fills)
                slot = (self.t - tau) % self.tau_max
                stale = self.grad_ring[slot, sl] if self.t >= tau else torch.zeros_like(g_cur[sl])
                st.grad[sl] = stale
                if self.needs_w:
                    w_stale = self.param_ring[slot, sl]
                    dw = st.master[sl] - w_stale
                    g = st.grad[sl]
                    if self.corrector == "dc_asgd":
                        st.grad[sl] = g + self.dc_lambda * g * g * dw
                    else:
                        self.v_ema[sl] = self.dc_beta2 * self.v_ema[sl] + (1 - self.dc_beta2) * g * g
                        st.grad[sl] = g + self.dc_lambda * self.v_ema[sl] * dw
            slot = self.t % self.tau_max
            self.grad_ring[slot] = g_cur
            if self.needs_w:
                self.param_ring[slot] = st.master
        if self.m_raw is not None:
            self.m_raw.mul_(self.pred_beta).add_(st.grad * grad_scale, alpha=1 - self.pred_beta)
        before = st.master.clone()
        self.inner.step(grad_scale=grad_scale, zero_grad=False)
        upd = st.master - before
        if self.damp != 1.0:
            st.master.copy_(before + self.damp * upd)
            upd = upd * self.damp
            st.sync_compute()
        self.last_update.copy_(upd)
        self.t += 1
        if zero_grad:
            st.zero_grad()

    # --------------------------------------------------------------------- forward predictor
    def has_forward_predictor(self) -> bool:
        return self.corrector in FORWARD_PRED

    @torch.no_grad()
    def offset(self) -> torch.Tensor:
        """Per-element forward offset (w_hat = w + offset)."""
        st = self.store
        out = torch.zeros_like(st.master)
        for info in st.infos:
            h = self.taus[info.name] * self.pred_scale
            if h == 0:
                continue
            sl = slice(info.offset, info.offset + info.numel)
            u = self.last_update[sl]
            if self.corrector == "weight_pred":
                out[sl] = h * u
                continue
            m = self.m_raw[sl]
            descent = -m / _rms(m)
            base = h * descent * _rms(u)
            if self.corrector == "wp_cautious":
                keep = (descent * u > 0).float()
                base = base * keep / (keep.mean() + EPS)
            elif self.corrector == "wp_confidence":
                cos = (descent * u).sum() / (_rms(descent) * _rms(u) * descent.numel())
                base = base * torch.clamp(cos, min=0.0)
            elif self.corrector == "wp_trust":
                cap = self.trust * _rms(st.master[sl])
                base = base * torch.clamp(cap / _rms(base), max=1.0)
            out[sl] = base
        return out

    @torch.no_grad()
    def apply_forward_offset(self) -> None:
        """Move the weights the forward reads to ``w + offset`` (undo with ``restore_weights``)."""
        if not self.has_forward_predictor():
            return
        st = self.store
        self._offset_backup = st.master.clone()
        st.master.add_(self.offset())
        st.sync_compute()

    @torch.no_grad()
    def restore_weights(self) -> None:
        if self._offset_backup is None:
            return
        st = self.store
        st.master.copy_(self._offset_backup)
        st.sync_compute()
        self._offset_backup = None


@dataclass(frozen=True)
class _DelayMixin:
    tau: int = 0
    corrector: str = "none"
    dc_lambda: float = 1.0
    dc_beta2: float = 0.99
    pred_scale: float = 1.0
    lr_damp: float = 1.0
    pred_beta: float = 0.95
    trust: float = 0.01
    num_stages: int = 0
    num_layers: int = 0

    def build(self, store, num_train_steps: int):
        from .fused import FusedOptimizer

        inner = FusedOptimizer(store, self, num_train_steps)
        leaf_tau = grug_stage_tau(self.num_layers, self.num_stages) if self.num_stages > 0 else None
        return DelayedOptimizer(inner, store, tau=self.tau, corrector=self.corrector, dc_lambda=self.dc_lambda,
                                dc_beta2=self.dc_beta2, lr_damp=self.lr_damp, pred_beta=self.pred_beta,
                                pred_scale=self.pred_scale, trust=self.trust, leaf_tau=leaf_tau)


@register("grug_moe_adamh_delayed")
@dataclass(frozen=True)
class DelayedGrugMoeAdamHConfig(_DelayMixin, GrugMoeAdamHConfig):
    """``grug_moe_adamh_v2`` behind the delayed-gradient wrapper."""


@register("grug_muon_delayed")
@dataclass(frozen=True)
class DelayedGrugMuonConfig(_DelayMixin, MuonConfig):
    """Muon behind the delayed-gradient wrapper."""
