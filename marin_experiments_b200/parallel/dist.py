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
        """Mean-all-reduce the gradients of replicated parameters (bucketed over the flat buffer).

        Expert shards already hold the sum over every rank's tokens of per-rank mean-loss gradients;
        dividing by the batch-group size turns that into the gradient of the global mean loss."""
        if self.world == 1:
            return
        st = trainer.store
        for info in self._sharded:
            g = st.grad[info.offset: info.offset + info.numel]
            if self.expert_dp_group is not None:  # replicas of this shard in other expert groups
                torch_dist.all_reduce(g, group=self.expert_dp_group)
            g.div_(self.world)
        # contiguous runs of replicated parameters in the flat buffer
        runs = []
        for info in self._replicated:
            s, e = info.offset, info.offset + info.numel
            if runs and runs[-1][1] >= s - 64:
                runs[-1][1] = e
            else:
                runs.append([s, e])
        limit = self.bucket_bytes // 4
        for s, e in runs:
            for c0 in range(s, e, limit):
                buf = st.grad[c0: min(e, c0 + limit)]
                torch_dist.all_reduce(buf, group=self.batch_group)
                buf.div_(self.world)


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
