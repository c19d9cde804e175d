"""Pipeline parallelism: stage models, P2P activation transfer and the schedule executor.

Topology: ``world = pp * ep`` ranks; rank ``r`` is stage ``r // ep``, expert-parallel index ``r % ep``.
Each stage holds ``num_layers / pp`` consecutive blocks (stage 0 also the embedding, the last stage
the final norm, head and loss) with its routed experts sharded over the stage's ``ep`` ranks, which
also split the batch (megagpt-speedrun/async_pipeline.py:442-662, grug-moe-pp/pipeline_zb.py:465-876).
Activations go stage to stage with ``isend``/``irecv`` (NCCL P2P over NVLink on GPUs, gloo on CPU);
forward and backward traffic use two separate process groups, so a stage's forward send and its
neighbour's backward send never wait behind each other on one communicator. ``SP_PP_TRANSPORT=null``
replaces the transfers with zeros (no traffic), the compute-only measurement of the reference's
null-transport switch (grug-moe-pp/pipeline_zb.py:115-118).

Modes:

* ``sync``: one optimizer step per batch after the pipeline flushes; the schedule is ``gpipe``,
  ``1f1b`` or ``zb`` (ZB-H1: the backward is split into the input-gradient pass B and the
  weight-gradient pass W, whose GEMMs are queued by ``ops.gemm.defer_weight_grads`` and run in the
  schedule's bubbles). Gradient clipping uses the global norm over all stages, so the update equals
  the unsplit model's (megagpt-speedrun/sync_pipeline.py:80-216 seeds the backward with 1/M; here
  the loss of every microbatch is scaled by 1/M).
* ``async``: 1F1B without flushes; every stage applies an optimizer update after each microbatch's
  backward, so stage ``s`` computes gradients on weights ``2 (P - 1 - s)`` updates stale
  (megagpt-speedrun/async_pipeline.py:442-662). Pair it with the delayed-gradient optimizers.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as tdist

from ..models.grug import apply_qb_betas, default_loss_weight
from ..ops import api as ops
from . import schedules as S


def stage_transport() -> str:
    """Stage-boundary transport named by the environment: ``SP_PP_TRANSPORT`` (``p2p`` or ``null``),
    or the reference benchmark's switch ``MOE_PP_NULL_XPORT=1`` (grug-moe-pp/pipeline_zb.py:118),
    which selects ``null``. An explicit ``SP_PP_TRANSPORT`` wins."""
    t = os.environ.get("SP_PP_TRANSPORT", "")
    if t:
        return t
    return "null" if os.environ.get("MOE_PP_NULL_XPORT", "0") not in ("", "0") else "p2p"


@dataclass
class PipelineTopology:
    pp: int
    ep: int
    rank: int
    world: int
    stage: int
    e: int
    stage_group: object
    chain_group: object
    fwd_group: object
    bwd_group: object

    @property
    def prev_rank(self) -> int:
        return (self.stage - 1) * self.ep + self.e

    @property
    def next_rank(self) -> int:
        return (self.stage + 1) * self.ep + self.e

    @property
    def is_first(self) -> bool:
        return self.stage == 0

    @property
    def is_last(self) -> bool:
        return self.stage == self.pp - 1


def init_topology(pp: int, ep: int = 1) -> PipelineTopology:
    """Create the stage, chain and P2P groups (every rank creates every group, in one order)."""
    rank, world = tdist.get_rank(), tdist.get_world_size()
    if pp * ep != world:
        raise ValueError(f"pp={pp} x ep={ep} != world size {world}")
    stage, e = rank // ep, rank % ep
    stage_group = chain_group = None
    for s in range(pp):
        g = tdist.new_group([s * ep + i for i in range(ep)])
        if s == stage:
            stage_group = g
    for i in range(ep):
        g = tdist.new_group([s * ep + i for s in range(pp)])
        if i == e:
            chain_group = g
    fwd = tdist.new_group(list(range(world)))
    bwd = tdist.new_group(list(range(world)))
    return PipelineTopology(pp, ep, rank, world, stage, e, stage_group, chain_group, fwd, bwd)


def stage_layers(num_layers: int, pp: int, stage: int) -> range:
    if num_layers % pp:
        raise ValueError(f"{num_layers} layers do not split evenly over {pp} stages")
    per = num_layers // pp
    return range(stage * per, (stage + 1) * per)


def _stage_dist(topo: PipelineTopology, backend: str, zero: bool = False):
    """The data/expert-parallel context inside one stage (its ``ep`` ranks): experts sharded over
    them, the other parameters replicated -- with ``zero``, the replicated parameters' optimizer
    state is sharded over the stage's ranks too (pipeline x ZeRO x expert parallelism)."""
    if topo.ep == 1:
        return None
    from .dist import DistContext
    from .fsdp import ZeroDistContext

    cls = ZeroDistContext if zero else DistContext
    return cls(rank=topo.e, world=topo.ep, ep_size=topo.ep, backend=backend, batch_group=topo.stage_group,
               ep_group=topo.stage_group, ep_rank=topo.e)


class PipelineTrainer:
    def __init__(self, cfg, topo: PipelineTopology, *, device, microbatches: int, schedule: str = "1f1b",
                 mode: str = "sync", num_train_steps: int | None = None, seed: int | None = None,
                 zero: bool = False):
        from ..train.trainer import Trainer

        self.cfg, self.topo, self.device = cfg, topo, torch.device(device)
        self.M, self.mode, self.schedule_name = microbatches, mode, schedule
        if mode not in ("sync", "async"):
            raise ValueError(f"unknown pipeline mode {mode}")
        mcfg = cfg.model
        self.layers = stage_layers(mcfg.num_layers, topo.pp, topo.stage)
        backend = "nccl" if self.device.type == "cuda" else "gloo"
        self.tr = Trainer(cfg, device=self.device, num_train_steps=num_train_steps, seed=seed,
                          dist=_stage_dist(topo, backend, zero),
                          model_kwargs=dict(layers=self.layers, with_embed=topo.is_first, with_head=topo.is_last))
        self.model = self.tr.model
        self.n_moe_total = mcfg.num_layers if mcfg.is_moe else 0
        if mode == "sync" and topo.pp > 1:
            self._chain_clip()
        self.act_dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.step = 0
        self._async_state = None
        # Stage-boundary transport: "p2p" (isend / irecv, sends complete in the background) or "null"
        # (nothing is sent, receivers get zeros: a compute-only measurement). A blocking send is not
        # offered: under 1F1B two neighbours can each block in a send on a different communicator
        # while the other waits to receive, a cycle.
        self.transport = stage_transport()
        if self.transport not in ("p2p", "null"):
            raise ValueError(f"SP_PP_TRANSPORT must be p2p or null, got {self.transport!r}")
        if topo.ep > 1:
            from . import ep

            ep.set_inflight_microbatches(max_inflight(schedule, topo.pp, microbatches, mode))

    # --------------------------------------------------------------------------- helpers
    def _chain_clip(self) -> None:
        """Global-norm clipping across stages: sum the per-group squared norms over the chain."""
        opt = getattr(self.tr.opt, "inner", self.tr.opt)
        inner_hook = opt.norm_hook
        chain = self.topo.chain_group

        def hook(gnorm2, names):
            if inner_hook is not None:
                inner_hook(gnorm2, names)
            tdist.all_reduce(gnorm2, group=chain)

        opt.norm_hook = hook

    def _send(self, t, dst, group, pending):
        if self.transport == "null":
            return
        pending.append(tdist.isend(t.contiguous(), dst, group=group))

    def _recv(self, shape, src, group):
        if self.transport == "null":
            return torch.zeros(shape, dtype=self.act_dtype, device=self.device)
        buf = torch.empty(shape, dtype=self.act_dtype, device=self.device)
        tdist.irecv(buf, src, group=group).wait()
        return buf

    def _aux(self, stats):
        """This stage's share of the router losses (the unsplit model averages over all layers)."""
        c = self.cfg.model
        if not stats:
            return None
        n = self.n_moe_total
        zl = torch.stack([s.z_loss for s in stats]).sum()
        sp = torch.stack([s.sparsity for s in stats]).sum()
        aux = c.router_z_loss_coef * zl / n + c.sparsity_loss_coef * sp / n
        if c.aux_loss_coef:
            aux = aux + c.aux_loss_coef * torch.stack([s.lbl for s in stats]).sum() / n
        return aux

    def _forward(self, m, tok, seg, lw, mb, s, slot=None):
        """Forward of microbatch ``m`` (rows ``m*mb .. (m+1)*mb`` of ``tok``); its expert-parallel
        buffers are those of in-flight slot ``slot`` (default ``m``)."""
        topo = self.topo
        sl = slice(m * mb, (m + 1) * mb)
        segm = None if seg is None else seg[sl].reshape(-1)
        x_in = None
        if topo.is_first:
            h = self.model.embed(tok[sl])
        else:
            x_in = self._recv((mb * s, self.cfg.model.hidden_dim), topo.prev_rank, topo.fwd_group)
            x_in.requires_grad_(True)
            h = x_in
        from . import ep

        with ep.microbatch_slot(m if slot is None else slot):
            h, stats = self.model.body(h, mb, s, segm, self.tr.dp_group)
        aux = self._aux(stats)
        beta = torch.stack([st.beta for st in stats]).detach() if stats and all(st.beta is not None for st in stats) \
            else None
        loss = None
        if topo.is_last:
            labels = torch.cat([tok[sl][:, 1:], torch.zeros_like(tok[sl][:, :1])], dim=1).reshape(-1)
            w = lw[sl] if lw is not None else default_loss_weight(mb, s, self.device)
            ce = ops.cross_entropy(self.model.head_input(h), self.model.head_weight(), labels,
                                   w.reshape(-1).float(), z_weight=self.tr.z_loss_weight)
            loss = ce if aux is None else ce + aux
            return x_in, None, loss, ce.detach(), beta
        return x_in, h, aux, None, beta

    def _backward(self, rec, queue, pending):
        topo = self.topo
        x_in, h, obj, _, _ = rec
        from ..ops import gemm as G

        ctx = G.defer_weight_grads(queue) if queue is not None else _nullctx()
        with ctx:
            if topo.is_last:
                (obj / self.M).backward()
            else:
                g = self._recv(h.shape, topo.next_rank, topo.bwd_group)
                outs, grads = [h], [g]
                if obj is not None:
                    outs.append(obj)
                    grads.append(torch.full_like(obj, 1.0 / self.M))
                torch.autograd.backward(outs, grads)
        if not topo.is_first:
            self._send(x_in.grad.to(self.act_dtype), topo.prev_rank, topo.bwd_group, pending)

    # ------------------------------------------------------------------------------ sync
    def train_step(self, batch: dict) -> dict:
        """One synchronous pipeline step over ``M`` microbatches of this rank's batch shard."""
        if self.mode != "sync":
            raise RuntimeError("train_step is the sync-mode step; use run_async for async mode")
        from ..ops import cuda_fns  # noqa: F401

        tr, topo = self.tr, self.topo
        tok = batch["tokens"].to(self.device, non_blocking=True)
        seg = batch.get("segment_ids")
        seg = None if seg is None else seg.to(self.device, non_blocking=True)
        lw = batch.get("loss_weight")
        lw = None if lw is None else lw.to(self.device, non_blocking=True)
        b, s = tok.shape
        if b % self.M:
            raise ValueError(f"batch {b} not divisible into {self.M} microbatches")
        mb = b // self.M
        if tr.pending_qb is not None and self.cfg.model.qb_balancing:
            apply_qb_betas(self.model, tr.pending_qb)
        if self.device.type == "cuda":
            cuda_fns.set_loss_grad_scale(1.0 / self.M)
        sched = S.SCHEDULES[self.schedule_name](topo.pp, self.M)[topo.stage]
        split = self.schedule_name == "zb"
        recs, queues, pending = {}, {}, []
        ce_sum = torch.zeros((), device=self.device)
        beta_sum = None
        for kind, m in sched:
            if kind == "F":
                rec = self._forward(m, tok, seg, lw, mb, s)
                recs[m] = rec
                if rec[1] is not None:
                    self._send(rec[1].detach(), topo.next_rank, topo.fwd_group, pending)
                if rec[3] is not None:
                    ce_sum = ce_sum + rec[3]
                if rec[4] is not None:
                    beta_sum = rec[4] if beta_sum is None else beta_sum + rec[4]
            elif kind == "B":
                queues[m] = [] if split else None
                self._backward(recs[m], queues[m], pending)
                if not split:
                    recs.pop(m)
            else:  # W
                from ..ops import gemm as G

                G.run_weight_grads(queues.pop(m))
                recs.pop(m, None)
        for p in pending:
            p.wait()
        if tr.dist is not None:
            tr.dist.grad_sync(tr)
        tr.opt.step()
        if tr.dist is not None and hasattr(tr.dist, "post_step"):
            tr.dist.post_step(tr)
        if beta_sum is not None:
            tr.pending_qb = beta_sum / self.M
        if tr.ema is not None:
            tr.ema.mul_(tr.ema_beta).add_(tr.store.master, alpha=1 - tr.ema_beta)
        tr.step += 1
        self.step += 1
        out = {}
        if topo.is_last:
            out["train/cross_entropy_loss"] = ce_sum / self.M
        return out

    # ----------------------------------------------------------------------------- async
    def _weights_used_by_forward(self):
        """Weight stashing for async mode: the backward of a microbatch must see the weights its
        forward saw (as a vjp closure does), while the optimizer keeps updating the live weights.
        On CPU the autograd graph saves parameter views, so saved tensors that alias the fp32 store
        are cloned when saved; on GPU the kernels read the bf16 compute buffer (and fp32 vector
        params) by reference, so a snapshot of those is taken here and swapped in around backward."""
        st = self.tr.store
        if self.device.type != "cuda":
            master_ptr = st.master.untyped_storage().data_ptr()

            def pack(t):
                if t.device.type == "cpu" and t.untyped_storage().data_ptr() == master_ptr:
                    return t.detach().clone()
                return t

            return torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t), None
        vec = [i for i in st.infos if i.ndim < 2]
        snap = (st.compute.clone(), [st.master[i.offset:i.offset + i.numel].clone() for i in vec], vec)
        return _nullctx(), snap

    def _swap_in(self, snap):
        st = self.tr.store
        comp, vecs, infos = snap
        live = (st.compute.clone(), [st.master[i.offset:i.offset + i.numel].clone() for i in infos], infos)
        st.compute.copy_(comp)
        for i, v in zip(infos, vecs):
            st.master[i.offset:i.offset + i.numel].copy_(v)
        return live

    def run_async(self, batches, n_ticks: int, as_tensors: bool = False) -> list:
        """Async 1F1B without flush over a stream of microbatches (each ``batches`` item is one
        microbatch). Stage ``s`` keeps ``P - 1 - s`` forwards in flight and updates its weights after
        every backward; each backward uses the weights of its own forward. Returns the last stage's
        per-microbatch losses (device tensors with ``as_tensors``, else floats)."""
        if self.mode != "async":
            raise RuntimeError("run_async needs mode='async'")
        from ..ops import cuda_fns  # noqa: F401

        tr, topo = self.tr, self.topo
        warm = topo.pp - 1 - topo.stage
        if self.device.type == "cuda":
            cuda_fns.set_loss_grad_scale(1.0)
        saveM, self.M = self.M, 1
        inflight, losses, pending = [], [], []
        it = iter(batches)
        try:
            for tick in range(n_ticks + warm):
                if tick < n_ticks:
                    bt = next(it)
                    tok = bt["tokens"].to(self.device, non_blocking=True)
                    seg = bt.get("segment_ids")
                    seg = None if seg is None else seg.to(self.device, non_blocking=True)
                    lw = bt.get("loss_weight")
                    lw = None if lw is None else lw.to(self.device, non_blocking=True)
                    if tr.pending_qb is not None and self.cfg.model.qb_balancing:
                        apply_qb_betas(self.model, tr.pending_qb)
                    hooks, snap = self._weights_used_by_forward()
                    with hooks:
                        rec = self._forward(0, tok, seg, lw, tok.shape[0], tok.shape[1], slot=tick)
                    if rec[1] is not None:
                        self._send(rec[1].detach(), topo.next_rank, topo.fwd_group, pending)
                    if rec[3] is not None:
                        losses.append(rec[3])
                    if rec[4] is not None:
                        tr.pending_qb = rec[4]
                    inflight.append((rec, snap))
                if tick >= warm and inflight:
                    rec, snap = inflight.pop(0)
                    live = self._swap_in(snap) if snap is not None else None
                    self._backward(rec, None, pending)
                    if live is not None:
                        self._swap_in(live)
                    if tr.dist is not None:
                        tr.dist.grad_sync(tr)
                    tr.opt.step()
                    if tr.dist is not None and hasattr(tr.dist, "post_step"):
                        tr.dist.post_step(tr)
                    tr.step += 1
            for p in pending:
                p.wait()
        finally:
            self.M = saveM
        return losses if as_tensors else [float(x) for x in losses]


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def max_inflight(schedule: str, pp: int, microbatches: int, mode: str = "sync") -> int:
    """Most microbatches any stage holds between their forward and backward: GPipe holds all ``M``,
    1F1B / ZB-H1 up to ``P``; the async no-flush mode ``P - s`` at stage s (``P`` at most)."""
    if mode == "async":
        return pp
    best = 1
    for stage_sched in S.SCHEDULES[schedule](pp, microbatches):
        live = 0
        for kind, _ in stage_sched:
            if kind == "F":
                live += 1
                best = max(best, live)
            elif kind == "B":
                live -= 1
    return best


def async_stage_delay(pp: int, stage: int) -> int:
    """Weight staleness (in updates) of stage ``stage`` under async 1F1B: ``2 (P - 1 - s)``."""
    return 2 * (pp - 1 - stage)


def bubble_fraction(schedule: str, pp: int, microbatches: int) -> float:
    sched = S.SCHEDULES[schedule](pp, microbatches)
    if schedule == "zb":
        return S.simulate(sched, 1.0, 1.0, 1.0)["bubble"]
    return S.simulate(sched, 1.0, 2.0)["bubble"]

