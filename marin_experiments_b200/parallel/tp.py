"""Tensor (model-axis) parallelism for attention heads and dense MLPs (megagpt-speedrun/model.py:247-275;
``SP_TP``, megagpt-speedrun/launch.py:261-262).

Rank ``r`` of a TP group of size ``n`` holds heads ``[r H/n, (r+1) H/n)`` of every attention layer
(its rows of ``w_qkv`` and ``attn_gate``, its columns of ``w_o``) and hidden units
``[r I/n, (r+1) I/n)`` of every dense / shared-expert MLP (its 128-row block pairs of the
interleaved ``w_gate_up``, its columns of ``w_down``). A TP block computes

    y = x + reduce(sublayer_local(copy(norm(x))))

where ``copy`` is the identity forward / all-reduce backward and ``reduce`` the all-reduce forward
/ identity backward (the column-parallel / row-parallel pair), so every rank keeps an identical
residual stream and identical gradients of the replicated parameters. Routed experts are not
TP-sharded (they are sharded over the expert axis instead). Global gradient-norm clipping sums the
TP-sharded parameters' squares over the group (``tp_norm_hook``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as tdist


@dataclass(frozen=True)
class TPInfo:
    rank: int
    size: int
    group: object = None


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        tdist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        y = x.contiguous().clone()
        tdist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_tp(x, tp: TPInfo | None):
    return x if tp is None or tp.size == 1 else _CopyToTP.apply(x, tp.group)


def reduce_from_tp(x, tp: TPInfo | None):
    return x if tp is None or tp.size == 1 else _ReduceFromTP.apply(x, tp.group)


# ------------------------------------------------------------------------------ shard layout
def local_counts(cfg, tp: TPInfo | None) -> tuple[int, int]:
    """(query heads, kv heads) held by this TP rank."""
    if tp is None or tp.size == 1:
        return cfg.num_heads, cfg.num_kv_heads
    if cfg.num_heads % tp.size or cfg.num_kv_heads % tp.size:
        raise ValueError(f"heads {cfg.num_heads}/{cfg.num_kv_heads} not divisible by tp={tp.size}")
    return cfg.num_heads // tp.size, cfg.num_kv_heads // tp.size


def local_inter(inter: int, tp: TPInfo | None, glu: bool = True) -> int:
    if tp is None or tp.size == 1:
        return inter
    if inter % tp.size or (glu and (inter // tp.size) % 128):
        raise ValueError(f"intermediate {inter} does not split into tp={tp.size} shards of 128-row blocks")
    return inter // tp.size


def shard(leaf: str, full: torch.Tensor, module, tp: TPInfo) -> torch.Tensor:
    """This rank's slice of a full-size parameter (used to initialise TP shards consistently with
    the unsplit model)."""
    r, n = tp.rank, tp.size
    if leaf == "w_qkv":
        c = module.cfg
        hd = c.inferred_head_dim
        nq, nk = c.num_heads * hd, c.num_kv_heads * hd
        q, k, v = full[:nq], full[nq:nq + nk], full[nq + nk:]
        return torch.cat([q.chunk(n)[r], k.chunk(n)[r], v.chunk(n)[r]], 0)
    if leaf == "attn_gate":
        return full.chunk(n, 0)[r]
    if leaf == "w_o":
        return full.chunk(n, 1)[r]
    if leaf == "w_gate_up":
        return full.chunk(n, 0)[r]  # contiguous 128-row block pairs in the interleaved layout
    if leaf == "w_down":
        return full.chunk(n, 1)[r]
    raise KeyError(leaf)


def full_shape(leaf: str, local: tuple, module, tp: TPInfo) -> tuple:
    n = tp.size
    if leaf in ("w_qkv", "attn_gate", "w_gate_up"):
        return (local[0] * n,) + tuple(local[1:])
    if leaf in ("w_o", "w_down"):
        return (local[0], local[1] * n)
    raise KeyError(leaf)


def setup_tp_optimizer(trainer, tp: TPInfo) -> None:
    """Make the fused optimizer see whole matrices: per-group squared gradient norms and the AdamH
    matrix sums of TP-sharded parameters are summed over the TP group (replicated parameters are
    identical on every rank and counted once), so the update equals the unsplit model's."""
    if tp is None or tp.size == 1:
        return
    tp_norm_hook(trainer, tp)
    opt = getattr(trainer.opt, "inner", trainer.opt)
    ids = opt.matrix_ids(lambda i: getattr(i, "tp_sharded", False))
    if not ids:
        return
    idx_cache = {}

    def mat_hook(sums):
        idx = idx_cache.get(sums.device)
        if idx is None:
            idx = idx_cache[sums.device] = torch.tensor(ids, dtype=torch.long, device=sums.device)
        part = sums.index_select(0, idx)
        tdist.all_reduce(part, group=tp.group)
        sums.index_copy_(0, idx, part)

    opt.mat_hook = mat_hook


def tp_norm_hook(trainer, tp: TPInfo):
    """Norm hook for the fused optimizer: per group, the squares of TP-sharded gradients are summed
    over the TP group (replicated ones are identical on every rank and counted once)."""
    opt = getattr(trainer.opt, "inner", trainer.opt)
    st = trainer.store
    sharded = {i.name for i in st.infos if getattr(i, "tp_sharded", False)}

    def hook(gnorm2, names):
        for gi, n in enumerate(names):
            part = torch.zeros((), dtype=torch.float64, device=gnorm2.device)
            for info in opt.groups[n]["infos"]:
                if info.name in sharded:
                    part += st.grad[info.offset: info.offset + info.numel].double().pow(2).sum().to(gnorm2.device)
            tot = part.clone()
            tdist.all_reduce(tot, group=tp.group)
            gnorm2[gi] = gnorm2[gi] - part + tot

    opt.norm_hook = hook
