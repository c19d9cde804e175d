"""Process groups and gradient synchronisation.

One process per GPU (``torch.distributed`` with NCCL on GPUs, gloo on CPU). The mesh is the
reference's ``(replica, data, expert, model)`` (megagpt-speedrun/model.py:84-105) restricted to what
the B200 build uses: every rank holds a batch shard; routed experts are sharded over the ``expert``
group (``ep_size`` ranks); everything else is replicated over the batch group and its gradients are
all-reduced (mean). Per-group squared gradient norms of expert-sharded optimizer groups are summed
over the expert group before clipping.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as torch_dist

# Gradient-sync timing: while installed (``dp_timing``), each ``grad_sync`` records CUDA events on
# the training stream around its part of the step -- the wait for reductions still running on the
# gradient stream plus the reductions left to do -- i.e. the data-parallel communication the step
# does not hide behind backward.
_DP_TIMING: list | None = None


class dp_timing:
    """``with dp_timing() as t: ...; t.ms()`` -- device milliseconds the training stream spent in
    gradient synchronisation inside the block."""

    def __enter__(self):
        global _DP_TIMING
        self.pairs = []
        _DP_TIMING = self.pairs
        return self

    def __exit__(self, *exc):
        global _DP_TIMING
        _DP_TIMING = None
        return False

    def ms(self) -> float:
        torch.cuda.synchronize()
        return float(sum(a.elapsed_time(b) for a, b in self.pairs))


def _dp_mark():
    if _DP_TIMING is None or not torch.cuda.is_available():
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    return ev


def _dp_span(start):
    if start is not None and _DP_TIMING is not None:
        _DP_TIMING.append((start, _dp_mark()))


@dataclass
class DistContext:
    rank: int
    world: int
    ep_size: int
    backend: str
    batch_group: object = None
    ep_group: object = None
    ep_rank: int = 0
    bucket_bytes: int = 256 << 20
    # ranks holding the same expert shard (one per expert-parallel group); None when ep == world
    expert_dp_group: object = None
    _armed: bool = False
    _launched: set = None

    def local_expert_range(self, num_experts: int) -> tuple[int, int]:
        if num_experts % self.ep_size:
            raise ValueError(f"num_experts={num_experts} must be divisible by ep_size={self.ep_size}")
        per = num_experts // self.ep_size
        return self.ep_rank * per, (self.ep_rank + 1) * per

    # ------------------------------------------------------------------ hooks used by Trainer
    def setup_model(self, trainer) -> None:
        from ..models.grug import MoEMLP

        if self.ep_size > 1:
            for blk in trainer.model.blocks:
                if isinstance(blk.mlp, MoEMLP):
                    blk.mlp.ep_group = self.ep_group
        # replicated parameters start identical on every rank
        st = trainer.store
        if self.world > 1:
            src = torch_dist.get_global_rank(self.batch_group, 0) if self.batch_group is not None else 0
            for info in st.infos:
                if info.sharded_over is None or self.ep_size == 1:
                    torch_dist.broadcast(st.master_view(info), src=src, group=self.batch_group)
            st.sync_compute()
        # expert weights are shards only under expert parallelism; with ep_size 1 they are replicated
        sharded = (lambda i: i.sharded_over is not None and self.ep_size > 1)
        self._replicated = [i for i in st.infos if not sharded(i) and i.trainable]
        self._sharded = [i for i in st.infos if sharded(i) and i.trainable]
        self.enable_overlap(trainer)

    def setup_optimizer(self, trainer) -> None:
        opt = getattr(trainer.opt, "inner", trainer.opt)
        sharded_groups = set()
        for name, g in opt.groups.items():
            if any(i.sharded_over == "expert" for i in g["infos"]):
                sharded_groups.add(name)
        if not sharded_groups or self.ep_size == 1:
            return
        ep_group = self.ep_group
        names_sharded = sharded_groups

        def norm_hook(gnorm2: torch.Tensor, names: list[str]) -> None:
            # expert-sharded groups: every rank holds different experts -> sum their squares. The
            # replicated members of such a group are counted ep_size times, so subtract the excess.
            opt_ = opt
            st = trainer.store
            for gi, n in enumerate(names):
                if n not in names_sharded:
                    continue
                rep = torch.zeros((), dtype=torch.float64, device=gnorm2.device)
                for info in opt_.groups[n]["infos"]:
                    if info.sharded_over is None:
                        g = st.grad[info.offset: info.offset + info.numel]
                        rep += (g.double() ** 2).sum()
                local_sh = gnorm2[gi] - rep
                tot = local_sh.clone().to(gnorm2.device)
                torch_dist.all_reduce(tot, group=ep_group)
                gnorm2[gi] = tot + rep

        opt.norm_hook = norm_hook

    def grad_sync(self, trainer) -> None:
        t0 = _dp_mark()
        self._grad_sync(trainer)
        _dp_span(t0)

    def _grad_sync(self, trainer) -> None:
        """Mean-all-reduce the gradients of replicated parameters (bucketed over the flat buffer).

        Expert shards already hold the sum over every rank's tokens of per-rank mean-loss gradients;
        dividing by the batch-group size turns that into the gradient of the global mean loss.

        With overlap armed for the step's last microbatch (``arm_overlap``), the ranges of the
        final norm / head and of every block were already all-reduced on the gradient stream as
        backward finished them; this joins that stream and reduces only what is left."""
        if self.world == 1:
            return
        st = trainer.store
        for info in self._sharded:
            g = st.grad[info.offset: info.offset + info.numel]
            if self.expert_dp_group is not None:  # replicas of this shard in other expert groups
                torch_dist.all_reduce(g, group=self.expert_dp_group)
            g.div_(self.world)
        runs = _runs(self._replicated)
        if self._armed:
            torch.cuda.current_stream().wait_stream(self._grad_stream)
            runs = _subtract(runs, sorted(self._launched))
            self._armed, self._launched = False, set()
        for s, e in runs:
            self._reduce_run(st, s, e, self.batch_group)

    # ---------------------------------------------------------------- overlap with backward
    # Per-segment hooks: a segment is a module (the final norm, then every block, in the order
    # backward finishes them) and the replicated flat-buffer runs of its parameters. A tensor hook
    # on the segment's input fires when backward has issued every kernel that writes the segment's
    # weight gradients (they precede the input gradient in the graph); on the step's last
    # microbatch the hook makes the gradient stream wait for the training stream and all-reduces
    # the segment's runs there, on a communicator of its own, while backward continues.
    supports_overlap = True  # a context whose grad_sync is not this one's turns it off

    def enable_overlap(self, trainer) -> None:
        if (not self.supports_overlap or self.world == 1 or self.backend != "nccl"
                or os.environ.get("MXK_DP_OVERLAP", "1") == "0"):
            return
        model, st = trainer.model, trainer.store
        ranks = list(range(self.world)) if self.batch_group is torch_dist.group.WORLD else None
        self._grad_group = torch_dist.new_group(ranks) if ranks is not None else self.batch_group
        self._grad_stream = torch.cuda.Stream(device=st.device)
        rep = {i.name: i for i in self._replicated}
        mods = []
        if getattr(model, "final_norm", None) is not None:
            tail = [n for n in rep if n.startswith(("final_norm.", "head_down", "output_proj"))]
            mods.append((model.final_norm, tail))
        for j, blk in enumerate(getattr(model, "blocks", [])):
            mods.append((blk, [n for n in rep if n.startswith(f"blocks.{j}.")]))
        for mod, names in mods:
            runs = [tuple(r) for r in _runs([rep[n] for n in names])]
            if runs:
                mod.register_forward_pre_hook(self._pre_hook(runs, st))
        self._overlap_on = True

    def arm_overlap(self) -> None:
        """Called before the step's last microbatch: its backward launches the segment reductions."""
        if getattr(self, "_overlap_on", False):
            self._armed, self._launched = True, set()

    def _pre_hook(self, runs, st):
        def pre(mod, args):
            if not (self._armed and torch.is_grad_enabled()):
                return None
            x = args[0]
            if torch.is_tensor(x) and x.requires_grad:
                x.register_hook(lambda g: self._launch(runs, st))
            return None
        return pre

    def _launch(self, runs, st):
        if not self._armed or all(r in self._launched for r in runs):
            return None
        side = self._grad_stream
        side.wait_stream(torch.cuda.current_stream(st.device))
        with torch.cuda.stream(side):
            for s, e in runs:
                if (s, e) not in self._launched:
                    self._reduce_run(st, s, e, self._grad_group)
                    self._launched.add((s, e))
        return None

    def _reduce_run(self, st, s: int, e: int, group) -> None:
        """Mean over the group of ``grad[s:e]`` in bucket-sized pieces; ``MXK_DP_WIRE=bf16`` sends
        bf16 (half the bytes; the sum is rounded to bf16 once)."""
        limit = self.bucket_bytes // 4
        bf16 = os.environ.get("MXK_DP_WIRE", "fp32") == "bf16" and st.grad.is_cuda
        for c0 in range(s, e, limit):
            buf = st.grad[c0: min(e, c0 + limit)]
            if bf16:
                w = buf.to(torch.bfloat16)
                torch_dist.all_reduce(w, group=group)
                buf.copy_(w).div_(self.world)
            else:
                torch_dist.all_reduce(buf, group=group)
                buf.div_(self.world)


def _subtract(runs, done) -> list[list[int]]:
    """The parts of the ``[s, e)`` runs not covered by the sorted, disjoint ``done`` intervals."""
    out = []
    for s, e in runs:
        cur = s
        for ds, de in done:
            if de <= cur or ds >= e:
                continue
            if ds > cur:
                out.append([cur, ds])
            cur = max(cur, de)
        if cur < e:
            out.append([cur, e])
    return out


def _runs(infos) -> list[list[int]]:
    """Contiguous flat-buffer runs covering the parameters ``infos`` (gaps of alignment padding merged)."""
    runs = []
    for info in sorted(infos, key=lambda i: i.offset):
        s, e = info.offset, info.offset + info.numel
        if runs and runs[-1][1] >= s - 64:
            runs[-1][1] = max(runs[-1][1], e)
        else:
            runs.append([s, e])
    return runs


_CTX: DistContext | None = None


def init(ep_size: int | None = None, timeout_s: float = 600.0) -> DistContext:
    global _CTX
    if _CTX is not None:
        return _CTX
    backend = "nccl" if torch.cuda.is_available() else "gloo"
    if not torch_dist.is_initialized():
        torch_dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
    rank, world = torch_dist.get_rank(), torch_dist.get_world_size()
    ep = world if ep_size is None else ep_size
    if world % ep:
        raise ValueError(f"world size {world} not divisible by ep_size {ep}")
    batch_group = torch_dist.group.WORLD
    ep_group = batch_group
    ep_rank = rank % ep
    expert_dp = None
    if ep != world:
        for start in range(0, world, ep):
            ranks = list(range(start, start + ep))
            g = torch_dist.new_group(ranks)
            if rank in ranks:
                ep_group = g
        if ep > 1:
            for e in range(ep):
                ranks = list(range(e, world, ep))
                g = torch_dist.new_group(ranks)
                if rank in ranks:
                    expert_dp = g
    _CTX = DistContext(rank=rank, world=world, ep_size=ep, backend=backend, batch_group=batch_group,
                       ep_group=ep_group, ep_rank=ep_rank, expert_dp_group=expert_dp)
    return _CTX


def shutdown() -> None:
    global _CTX
    if torch_dist.is_initialized():
        torch_dist.barrier()
        torch_dist.destroy_process_group()
    _CTX = None
