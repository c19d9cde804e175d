"""Fully sharded data parallelism over the flat parameter store (ZeRO stage 2).

The reference shards every weight over the ``data`` mesh axis and lets XLA insert the parameter
all-gather and gradient reduce-scatter (megagpt-speedrun/model.py:247-250,340-342; explicit form in
grug-moe-pp/pipeline.py:434-480). Here the unit of sharding is the flat fp32 buffer of the
``ParamStore``: rank ``r`` owns the range ``[r * n / W, (r + 1) * n / W)``.

One step:

1. backward accumulates full-size fp32 gradients (bucketable, as in plain data parallelism);
2. ``grad_sync`` reduce-scatters them in place, so each rank holds the mean gradient of its range;
3. the fused optimizer updates only its range: the moments exist only for the range, the per-group
   squared gradient norms and the AdamH per-matrix sums ``(S_pp, S_pu, S_uu)`` are partial and
   all-reduced between the kernel's two passes (a few KB);
4. ``post_step`` all-gathers the updated fp32 range into every rank's master buffer and refreshes the
   bf16 compute copy.

Optimizer memory per rank drops from ``8 n`` to ``8 n / W`` bytes; the bytes on the wire equal a
gradient all-reduce. Experts are replicated (pure data parallelism); combine with expert parallelism
by sharding the replicated parameters only, which this context does not do.
"""

from __future__ import annotations

import torch
import torch.distributed as tdist

from .dist import DistContext


class ZeroDistContext(DistContext):
    supports_overlap = False  # the reduce-scatter runs once, after backward

    @property
    def store_pad(self) -> int:
        return 64 * self.world

    def shard_range(self, numel: int) -> tuple[int, int]:
        per = numel // self.world
        return self.rank * per, (self.rank + 1) * per

    def setup_model(self, trainer) -> None:
        if self.ep_size != 1:
            raise ValueError("ZeRO data parallelism replicates the experts (ep_size must be 1)")
        super().setup_model(trainer)
        st = trainer.store
        align = 64 * self.world
        if st.numel % align:
            raise ValueError(f"flat store size {st.numel} is not a multiple of {align}")

    def setup_optimizer(self, trainer) -> None:
        opt = getattr(trainer.opt, "inner", trainer.opt)
        lo, hi = self.shard_range(trainer.store.numel)
        opt.set_shard(lo, hi)
        group = self.batch_group

        def allreduce(t):
            tdist.all_reduce(t, group=group)

        opt.norm_hook = lambda g2, names: allreduce(g2)
        opt.mat_hook = allreduce
        self._shard = (lo, hi)

    def grad_sync(self, trainer) -> None:
        st = trainer.store
        lo, hi = self._shard
        if self.backend == "nccl":
            tdist.reduce_scatter_tensor(st.grad[lo:hi], st.grad, op=tdist.ReduceOp.SUM, group=self.batch_group)
        else:  # gloo has no reduce-scatter: all-reduce and keep the range
            tdist.all_reduce(st.grad, group=self.batch_group)
        st.grad[lo:hi].div_(self.world)

    def post_step(self, trainer) -> None:
        st = trainer.store
        lo, hi = self._shard
        if self.backend == "nccl":
            tdist.all_gather_into_tensor(st.master, st.master[lo:hi].clone(), group=self.batch_group)
        else:
            parts = list(st.master.chunk(self.world))
            tdist.all_gather(parts, st.master[lo:hi].clone(), group=self.batch_group)
            st.master.copy_(torch.cat(parts))
        st.sync_compute()


def init_zero(timeout_s: float = 600.0) -> ZeroDistContext:
    from . import dist as pdist

    base = pdist.init(ep_size=1, timeout_s=timeout_s)
    ctx = ZeroDistContext(rank=base.rank, world=base.world, ep_size=1, backend=base.backend,
                          batch_group=base.batch_group, ep_group=base.ep_group, ep_rank=0)
    pdist._CTX = ctx
    return ctx
