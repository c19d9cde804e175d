"""Fully sharded data parallelism over the flat parameter store (ZeRO stage 2), alone or composed
with expert parallelism.

The reference shards every weight over the ``data`` mesh axis and lets XLA insert the parameter
all-gather and gradient reduce-scatter (megagpt-speedrun/model.py:247-250,340-342; explicit form in
grug-moe-pp/pipeline.py:434-480), next to the ``expert`` axis that shards the routed experts
(megagpt-speedrun/model.py:245-251). Here the unit of sharding is the flat fp32 buffer of the
``ParamStore``.

* Pure data parallelism (``ep_size == 1``): rank ``r`` owns ``[r * n / W, (r + 1) * n / W)`` of the
  whole buffer.
* With expert parallelism (``ep_size == W``): the store lays the routed experts out last
  (``ParamStore(expert_last=True)``); the replicated prefix ``[0, R)`` is sharded over the ranks as
  above, and each rank keeps the full optimizer state of its own experts ``[R, n)`` -- those are
  already distinct on every rank.

One step:

1. backward accumulates full-size fp32 gradients (bucketable, as in plain data parallelism);
2. ``grad_sync`` reduce-scatters the sharded region in place, so each rank holds the mean gradient
   of its range; expert gradients (already summed over every source rank's tokens) are scaled to
   the mean;
3. the fused optimizer updates only its ranges: the moments exist only for them, the per-group
   squared gradient norms and the AdamH per-matrix sums ``(S_pp, S_pu, S_uu)`` are partial and
   all-reduced between the kernel's two passes (a few KB) -- replicated matrices are split over
   the ranks' shards and summed; each expert matrix lives whole on its rank, whose sums are kept
   (the group norms sum over all ranks: every expert is counted once);
4. ``post_step`` all-gathers the updated fp32 shards into every rank's master buffer and refreshes
   the bf16 compute copy.

Optimizer memory per rank for the sharded region drops from ``8 n`` to ``8 n / W`` bytes; the
bytes on the wire equal a gradient all-reduce.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as tdist

from .dist import DistContext

# flag purposes of the peer-memory ZeRO exchanges (a heap of their own)
_RS_READY, _RS_DONE, _AG_READY = 4, 5, 6


class ZeroDistContext(DistContext):
    """On GPUs the gradient reduce-scatter and the parameter all-gather run as this framework's own
    kernels over peer memory (``MXK_ZERO_P2P``, on by default): the store's fp32 master and gradient
    buffers live in a symmetric heap (every rank maps every other rank's), each rank sums its shard
    of everyone's gradients straight from their buffers with the mean applied in the same pass, and
    pulls the other ranks' updated shards into its masters while writing the bf16 copy. Release /
    acquire flags order the passes: gradients complete before anyone reads them, nobody clears its
    gradients before every rank has read them, shards updated before anyone pulls them."""

    supports_overlap = False  # the reduce-scatter runs once, after backward

    @property
    def p2p(self) -> bool:
        return self.backend == "nccl" and os.environ.get("MXK_ZERO_P2P", "1") == "1"

    @property
    def store_alloc(self):
        if not self.p2p:
            return None

        def alloc(numel: int):
            from .symm import heap_for

            dev = torch.device("cuda", torch.cuda.current_device())
            nbytes = 4 * numel
            heap = heap_for(self.batch_group, dev, 2 * nbytes + (2 << 20), name="zero")
            self._heap = heap
            self._master_off = heap.alloc("zero_master", nbytes)
            self._grad_off = heap.alloc("zero_grad", nbytes)
            return (heap.tensor(self._master_off, (numel,), torch.float32),
                    heap.tensor(self._grad_off, (numel,), torch.float32))

        return alloc

    def _flag(self, purpose: int) -> None:
        from ..ops._ext import err_flag, ext

        h = self._heap
        e = h.next_epoch(purpose)
        ext().ep_signal(h.peers, h.my, 0, purpose, e)
        ext().ep_wait(h.peers, h.my, 0, purpose, e, err_flag(h.device))

    @property
    def store_pad(self) -> int:
        return 64 * self.world

    @property
    def expert_last(self) -> bool:
        return self.ep_size > 1

    def _sharded_end(self, store) -> int:
        """End of the region sharded over the ranks: the replicated prefix (experts after it)."""
        return store.expert_start if self.ep_size > 1 else store.numel

    def shard_range(self, numel: int) -> tuple[int, int]:
        per = numel // self.world
        return self.rank * per, (self.rank + 1) * per

    def setup_model(self, trainer) -> None:
        if self.ep_size not in (1, self.world):
            raise ValueError("ZeRO shards the replicated parameters over all ranks and keeps each rank's "
                             "experts local: ep_size must be 1 or the world size")
        super().setup_model(trainer)
        st = trainer.store
        align = 64 * self.world
        if self._sharded_end(st) % align:
            raise ValueError(f"sharded region {self._sharded_end(st)} is not a multiple of {align}")

    def setup_optimizer(self, trainer) -> None:
        opt = getattr(trainer.opt, "inner", trainer.opt)
        st = trainer.store
        end = self._sharded_end(st)
        lo, hi = self.shard_range(end)
        extra = [(end, st.numel)] if self.ep_size > 1 and st.numel > end else []
        opt.set_shard(lo, hi, *extra)
        group = self.batch_group

        def allreduce(t):
            tdist.all_reduce(t, group=group)

        # AdamH matrix sums: replicated matrices are split over the ranks' shards (sum them); an
        # expert matrix id names a different expert on every rank and is complete locally.
        local = opt.matrix_ids(lambda i: i.sharded_over == "expert") if self.ep_size > 1 else []
        local_idx = torch.tensor(local, dtype=torch.long, device=st.device) if local else None

        def mat_hook(sums):
            if local_idx is None:
                allreduce(sums)
                return
            keep = sums.index_select(0, local_idx)
            allreduce(sums)
            sums.index_copy_(0, local_idx, keep)

        opt.norm_hook = lambda g2, names: allreduce(g2)
        opt.mat_hook = mat_hook
        self._shard = (lo, hi)
        self._end = end

    def grad_sync(self, trainer) -> None:
        st = trainer.store
        lo, hi = self._shard
        region = st.grad[: self._end]
        if getattr(self, "_heap", None) is not None:
            from ..ops._ext import ext

            self._flag(_RS_READY)  # every rank's gradients are complete
            ext().zero_rs(self._heap.peers, self._grad_off, lo, hi, st.grad, 1.0 / self.world)
            self._flag(_RS_DONE)  # every rank has read its shard of everyone's gradients
            if self._end < st.numel:
                st.grad[self._end:].div_(self.world)
            return
        if self.backend == "nccl":
            tdist.reduce_scatter_tensor(st.grad[lo:hi], region, op=tdist.ReduceOp.SUM, group=self.batch_group)
        else:  # gloo has no reduce-scatter: all-reduce and keep the range
            tdist.all_reduce(region, group=self.batch_group)
        st.grad[lo:hi].div_(self.world)
        if self._end < st.numel:  # this rank's experts: sum over all ranks' tokens -> mean
            st.grad[self._end:].div_(self.world)

    def post_step(self, trainer) -> None:
        st = trainer.store
        lo, hi = self._shard
        region = st.master[: self._end]
        if getattr(self, "_heap", None) is not None:
            from ..ops._ext import ext

            self._flag(_AG_READY)  # every rank's shard is updated
            ext().zero_ag(self._heap.peers, self._heap.my, self._master_off, hi - lo, self._end, st.master, st.compute)
            if self._end < st.numel:  # this rank's experts: their bf16 copy
                ext().cast_bf16(st.master[self._end:], st.compute[self._end:])
            return
        if self.backend == "nccl":
            tdist.all_gather_into_tensor(region, st.master[lo:hi].clone(), group=self.batch_group)
        else:
            parts = list(region.chunk(self.world))
            tdist.all_gather(parts, st.master[lo:hi].clone(), group=self.batch_group)
            region.copy_(torch.cat(parts))
        st.sync_compute()


def init_zero(timeout_s: float = 600.0, ep_size: int = 1) -> ZeroDistContext:
    """ZeRO data parallelism over every rank; ``ep_size`` = the world size also shards the routed
    experts over the ranks (expert parallelism)."""
    from . import dist as pdist

    base = pdist.init(ep_size=ep_size, timeout_s=timeout_s)
    ctx = ZeroDistContext(rank=base.rank, world=base.world, ep_size=base.ep_size, backend=base.backend,
                          batch_group=base.batch_group, ep_group=base.ep_group, ep_rank=base.ep_rank,
                          expert_dp_group=base.expert_dp_group)
    pdist._CTX = ctx
    return ctx
