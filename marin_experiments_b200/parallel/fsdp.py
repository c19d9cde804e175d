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

Muon orthogonalises whole matrices, so its matrices are not split: a rank's optimizer range is its
reduce-scatter range with each boundary moved forward past a Muon matrix that crosses it, and the
rank holding a matrix's first element owns its momentum and its Newton-Schulz step. The only extra
traffic is for the matrices that cross a boundary: after the reduce-scatter, each rank hands the
part of its range that belongs to an earlier rank's matrix to that owner (one small all-gather),
and after the step the owners hand the updated parameters back before the all-gather of the shards.
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
        spans = sorted((i.offset, (i.offset + i.numel + 3) // 4 * 4) for i in getattr(opt, "muon_infos", ())
                       if i.offset < end)
        self._end = end
        self._bounds = muon_bounds(spans, end, self.world)
        # exchange sizes: the longest foreign part (gradients to owners), the longest tail (parameters back)
        self._xg = max(b - a for a, b in map(self._foreign, range(self.world)))
        self._xp = max(b - a for a, b in map(self._outside, range(self.world)))
        opt.set_shard(self._bounds[self.rank], self._bounds[self.rank + 1], *extra)
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

    # ------------------------------------------------------------------ Muon matrices across shards
    def _foreign(self, q: int) -> tuple[int, int]:
        """Part of rank q's reduce-scatter range that an earlier rank's Muon matrix owns."""
        per = self._end // self.world
        lo, hi = q * per, (q + 1) * per
        return lo, max(lo, min(self._bounds[q], hi))

    def _outside(self, r: int) -> tuple[int, int]:
        """Part of rank r's optimizer range beyond its reduce-scatter range (matrix tails)."""
        per = self._end // self.world
        a, b = max(self._bounds[r], (r + 1) * per), self._bounds[r + 1]
        return a, max(a, b)

    def _gather_pieces(self, src: torch.Tensor, span: tuple[int, int], size: int) -> torch.Tensor:
        piece = torch.zeros(size, dtype=src.dtype, device=src.device)
        piece[: span[1] - span[0]] = src[span[0]: span[1]]
        if self.backend == "nccl":
            out = torch.empty(self.world * size, dtype=src.dtype, device=src.device)
            tdist.all_gather_into_tensor(out, piece, group=self.batch_group)
            return out.view(self.world, size)
        parts = [torch.empty_like(piece) for _ in range(self.world)]
        tdist.all_gather(parts, piece, group=self.batch_group)
        return torch.stack(parts)

    def _muon_grads_to_owners(self, st) -> None:
        if not self._xg:
            return
        got = self._gather_pieces(st.grad, self._foreign(self.rank), self._xg)
        a, b = self._outside(self.rank)
        for q in range(self.rank + 1, self.world):
            f0, f1 = self._foreign(q)
            x0, x1 = max(a, f0), min(b, f1)
            if x1 > x0:
                st.grad[x0:x1] = got[q, x0 - f0: x1 - f0]

    def _muon_params_from_owners(self, st) -> None:
        if not self._xp:
            return
        got = self._gather_pieces(st.master, self._outside(self.rank), self._xp)
        f0, f1 = self._foreign(self.rank)
        for r in range(self.rank):
            a, b = self._outside(r)
            x0, x1 = max(a, f0), min(b, f1)
            if x1 > x0:
                st.master[x0:x1] = got[r, x0 - a: x1 - a]

    def _grad_sync(self, trainer) -> None:
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
            self._muon_grads_to_owners(st)
            return
        if self.backend == "nccl":
            tdist.reduce_scatter_tensor(st.grad[lo:hi], region, op=tdist.ReduceOp.SUM, group=self.batch_group)
        else:  # gloo has no reduce-scatter: all-reduce and keep the range
            tdist.all_reduce(region, group=self.batch_group)
        st.grad[lo:hi].div_(self.world)
        if self._end < st.numel:  # this rank's experts: sum over all ranks' tokens -> mean
            st.grad[self._end:].div_(self.world)
        self._muon_grads_to_owners(st)

    def post_step(self, trainer) -> None:
        from .dist import _dp_mark, _dp_span

        t0 = _dp_mark()
        self._post_step(trainer)
        _dp_span(t0)

    def _post_step(self, trainer) -> None:
        st = trainer.store
        lo, hi = self._shard
        region = st.master[: self._end]
        self._muon_params_from_owners(st)
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


def muon_bounds(spans: list[tuple[int, int]], end: int, world: int) -> list[int]:
    """Optimizer range boundaries ``[a_0 = 0, ..., a_W = end]``: the equal reduce-scatter
    boundaries, each moved forward to the end of a Muon matrix span ``[s, e)`` that contains it."""
    per = end // world
    out = []
    for r in range(world + 1):
        b = min(r * per, end) if r < world else end
        for s, e in spans:
            if s < b < e:
                b = e
        out.append(max(b, out[-1]) if out else b)
    return out


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
