"""Grug transformer: the dense Llama-style decoder and the QB-routed MoE decoder.

One definition covers
* the tiny-stories dense model (tiny-stories/model.py:58-226): embed -> N x (RMSNorm -> attention,
  RMSNorm -> MLP) -> RMSNorm -> untied head, ReLU or SwiGLU MLP;
* the grug MoE / megagpt-speedrun model (megagpt-speedrun/model.py:234-838): GatedNorm after every
  RMSNorm, QK-normed GQA attention with exclusive self-attention and a per-head gate, sliding
  local/global attention windows, a fp32 router with loss-free (QB) balancing, sigmoid combine
  weights, optional adaptive (variable-k) routing, routed SwiGLU experts plus a shared expert,
  and an optional factorised embedding.

Tokens are processed flattened (``[B*S, D]``). Parameters use the ``[out, in]`` layout and the
block-interleaved gate/up layout of ``ops.layout``. Expert-parallel sharding keeps only the
local experts' rows of ``w_gate_up``/``w_down`` on each rank (``local_experts``); the dispatch
across ranks is done by ``parallel.ep``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from ..config import GrugModelConfig
from ..ops import api as ops


def trunc_normal_(t: torch.Tensor, std: float, generator: torch.Generator | None = None) -> torch.Tensor:
    """std * truncated_normal(-3, 3) (megagpt-speedrun/model.py:841-842)."""
    with torch.no_grad():
        t.normal_(0.0, 1.0, generator=generator)
        t.clamp_(-3.0, 3.0)
        t.mul_(std)
    return t


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps


class GatedNorm(nn.Module):
    """x * sigmoid(silu(x W_down^T) W_up^T), rank ``r`` (megagpt-speedrun/model.py:306-328)."""

    def __init__(self, dim: int, rank: int):
        super().__init__()
        self.w_down = nn.Parameter(torch.empty(rank, dim))
        self.w_up = nn.Parameter(torch.empty(dim, rank))


class NormPair(nn.Module):
    """RMSNorm followed by an optional GatedNorm."""

    def __init__(self, cfg: GrugModelConfig):
        super().__init__()
        self.rms = RMSNorm(cfg.hidden_dim, cfg.layer_norm_eps)
        self.gated = GatedNorm(cfg.hidden_dim, cfg.gated_norm_rank) if cfg.gated_norm else None

    def forward(self, x):
        if self.gated is None:
            return ops.rms_gated_norm(x, self.rms.weight, self.rms.eps)
        return ops.rms_gated_norm(x, self.rms.weight, self.rms.eps, self.gated.w_down, self.gated.w_up)

    def with_residual(self, x):
        """``(norm(x), residual)`` -- see ``ops.rms_gated_norm_res``."""
        g = self.gated
        return ops.rms_gated_norm_res(x, self.rms.weight, self.rms.eps, None if g is None else g.w_down,
                                      None if g is None else g.w_up)


class Attention(nn.Module):
    tp_sharded_params = ("w_qkv", "attn_gate", "w_o")

    def __init__(self, cfg: GrugModelConfig, layer: int, tp=None):
        super().__init__()
        from ..parallel.tp import local_counts

        d, hd = cfg.hidden_dim, cfg.inferred_head_dim
        h, hkv = local_counts(cfg, tp)  # heads held by this tensor-parallel rank
        self.tp = tp
        # w_qkv rows: [q heads | k heads | v heads]; attn_gate rows follow it contiguously in the
        # parameter store so one GEMM produces q, k, v and the head-gate logits.
        self.w_qkv = nn.Parameter(torch.empty((h + 2 * hkv) * hd, d))
        self.attn_gate = nn.Parameter(torch.zeros(h, d)) if cfg.head_gate else None
        self.w_o = nn.Parameter(torch.empty(d, h * hd))
        self.window = cfg.layer_window(layer)
        self.cfg = cfg

    def forward(self, h, x, batch: int, seq: int, segment_ids=None):
        from ..parallel.tp import copy_to_tp, local_counts, reduce_from_tp

        c = self.cfg
        nh, nkv = local_counts(c, self.tp)
        shape = ops.AttnShape(batch, seq, nh, nkv, c.inferred_head_dim, window=self.window,
                              qk_mult=c.qk_mult, qk_norm=c.qk_norm, xsa=c.xsa, head_gate=c.head_gate,
                              rope_theta=c.rope.theta, llama3=_llama3(c))
        if self.tp is None or self.tp.size == 1:
            return ops.attention_block(h, x, self.w_qkv, self.attn_gate, self.w_o, shape, segment_ids)
        part = ops.attention_block(copy_to_tp(h, self.tp), torch.zeros_like(x), self.w_qkv, self.attn_gate,
                                   self.w_o, shape, segment_ids)
        return x + reduce_from_tp(part, self.tp)


def _llama3(c: GrugModelConfig):
    if not c.rope.llama3_scaling:
        return None
    r = c.rope
    return {"scaling_factor": r.scaling_factor, "low_freq_factor": r.low_freq_factor,
            "high_freq_factor": r.high_freq_factor, "original_max_position": r.original_max_position}


class DenseMLP(nn.Module):
    """SwiGLU (``glu``; blocked gate/up rows) or plain activation MLP."""

    tp_sharded_params = ("w_gate_up", "w_down")

    def __init__(self, dim: int, inter: int, glu: bool, act: str, tp=None):
        super().__init__()
        from ..parallel.tp import local_inter

        inter = local_inter(inter, tp, glu)
        self.w_gate_up = nn.Parameter(torch.empty((2 if glu else 1) * inter, dim))
        self.w_down = nn.Parameter(torch.empty(dim, inter))
        self.glu, self.act, self.tp = glu, act, tp

    def forward(self, h, residual=None):
        if self.tp is None or self.tp.size == 1:
            return ops.dense_mlp(h, self.w_gate_up, self.w_down, glu=self.glu, act=self.act, residual=residual)
        from ..parallel.tp import copy_to_tp, reduce_from_tp

        part = ops.dense_mlp(copy_to_tp(h, self.tp), self.w_gate_up, self.w_down, glu=self.glu, act=self.act)
        y = reduce_from_tp(part, self.tp)
        return y if residual is None else residual + y


@dataclass
class RouterStats:
    z_loss: torch.Tensor
    lbl: torch.Tensor
    sparsity: torch.Tensor
    counts: torch.Tensor
    entropy: torch.Tensor
    beta: torch.Tensor | None
    expected_active_frac: torch.Tensor
    realized_active_frac: torch.Tensor
    threshold: torch.Tensor


class MoEMLP(nn.Module):
    """QB-routed MoE with sigmoid combine weights (megagpt-speedrun/model.py:470-645)."""

    def __init__(self, cfg: GrugModelConfig, local_experts: tuple[int, int] | None = None):
        super().__init__()
        d, e, i = cfg.hidden_dim, cfg.num_experts, cfg.intermediate_dim
        lo, hi = local_experts if local_experts is not None else (0, e)
        self.expert_range = (lo, hi)
        self.router = nn.Parameter(torch.empty(e, d))
        self.router_bias = nn.Parameter(torch.zeros(e), requires_grad=False)
        self.router_threshold = nn.Parameter(torch.full((), -4.0))
        self.w_gate_up = nn.Parameter(torch.empty(hi - lo, 2 * i, d))
        self.w_down = nn.Parameter(torch.empty(hi - lo, d, i))
        self.cfg = cfg
        self.ep_group = None  # set by parallel.ep when experts are sharded
        self.layer_key = 0  # this layer's index (keys its expert-parallel receive buffers)

    def forward(self, h, residual=None, dp_group=None, logit_bias=None):
        c = self.cfg
        t = h.shape[0]
        world = 1
        if dp_group is not None:
            world = torch.distributed.get_world_size(dp_group)
        qb_count = max(1, t * c.num_experts_per_token // c.num_experts)
        r = ops.route(h, self.router, self.router_bias, c.num_experts_per_token, adaptive=c.adaptive_routing,
                      threshold=self.router_threshold, k_min=c.min_experts_per_token, temp=c.sparsity_temp,
                      qb_count=qb_count, need_beta=c.qb_balancing, logit_bias=logit_bias)
        beta = r.beta
        if beta is not None and world > 1:
            beta = beta.clone()
            torch.distributed.all_reduce(beta, group=dp_group)
            beta = beta / world
        cap = None
        if c.capacity_factor and c.capacity_factor > 0:
            cap = ops.capacity_for(t, c.num_experts_per_token, c.num_experts, c.capacity_factor)
        if self.ep_group is not None:
            from ..parallel import ep

            y = ep.moe_experts_ep(h, r, self.w_gate_up, self.w_down, cap, self.ep_group, residual=residual,
                                  layer=self.layer_key, n_layers=c.num_layers)
        else:
            y = ops.moe_experts(h, r, self.w_gate_up, self.w_down, capacity=cap, residual=residual)
        stats = RouterStats(r.z_loss, r.lbl, r.sparsity, r.counts, r.entropy, beta, r.expected_active,
                            r.realized_active, self.router_threshold.detach())
        return y, stats


class Block(nn.Module):
    def __init__(self, cfg: GrugModelConfig, layer: int, local_experts=None, tp=None):
        super().__init__()
        self.attn_norm = NormPair(cfg)
        self.attn = Attention(cfg, layer, tp)
        self.mlp_norm = NormPair(cfg)
        if cfg.is_moe:
            self.mlp = MoEMLP(cfg, local_experts)
            self.mlp.layer_key = layer
            self.shared = (DenseMLP(cfg.hidden_dim, cfg.shared_expert_intermediate_dim, True, "silu", tp)
                           if cfg.shared_expert_intermediate_dim > 0 else None)
        else:
            self.mlp = DenseMLP(cfg.hidden_dim, cfg.intermediate_dim, cfg.glu, cfg.mlp_activation, tp)
            self.shared = None
        self.cfg = cfg

    def forward(self, x, batch: int, seq: int, segment_ids=None, dp_group=None, logit_bias=None):
        """One block. Under ``remat_mode`` (megagpt-speedrun/model.py:760-769) the block runs inside
        ``torch.utils.checkpoint`` (non-reentrant: the saved tensors are dropped after the forward
        and the region is re-run when backward first needs them): ``recompute_all`` checkpoints the
        whole block, ``save_moe`` everything before the routed experts, whose activations (and
        token exchange, under expert parallelism) are kept. Every rank re-runs the same regions in
        the same order, so the exchanges inside a recomputed region stay matched across ranks."""
        mode = self.cfg.remat_mode
        if mode == "none" or not torch.is_grad_enabled():
            return self._forward(x, batch, seq, segment_ids, dp_group, logit_bias)
        from torch.utils.checkpoint import checkpoint

        if mode == "recompute_all" or not self.cfg.is_moe:
            return checkpoint(self._forward, x, batch, seq, segment_ids, dp_group, logit_bias, use_reentrant=False)
        overlap = self._shared_overlap(x)
        h, x, base = checkpoint(self._pre_moe, x, batch, seq, segment_ids, not overlap, use_reentrant=False)
        return self._moe(h, x, base, dp_group, logit_bias, overlap)

    def _shared_overlap(self, x) -> bool:
        if self.shared is None or self.shared.tp is not None or self.mlp.ep_group is None:
            return False
        from ..parallel import ep

        return ep.overlap_shared_enabled(x, self.mlp.ep_group)

    def _pre_moe(self, x, batch: int, seq: int, segment_ids, with_shared: bool):
        """Norms and attention (and the shared expert, unless it runs beside the routed experts):
        ``(h, residual, base)`` where ``base`` is the routed experts' residual input."""
        h, x = self.attn_norm.with_residual(x)
        x = self.attn(h, x, batch, seq, segment_ids)
        h, x = self.mlp_norm.with_residual(x)
        base = self.shared(h, residual=x) if (with_shared and self.shared is not None) else x
        return h, x, base

    def _moe(self, h, x, base, dp_group, logit_bias, overlap: bool):
        if overlap:
            from ..parallel import ep

            # shared expert on a side stream while the routed experts exchange tokens
            return ep.with_shared_overlap(
                h, self.shared, lambda: self.mlp(h, residual=x, dp_group=dp_group, logit_bias=logit_bias))
        return self.mlp(h, residual=base, dp_group=dp_group, logit_bias=logit_bias)

    def _forward(self, x, batch: int, seq: int, segment_ids=None, dp_group=None, logit_bias=None):
        if not self.cfg.is_moe:
            h, x = self.attn_norm.with_residual(x)
            x = self.attn(h, x, batch, seq, segment_ids)
            h, x = self.mlp_norm.with_residual(x)
            return self.mlp(h, residual=x), None
        overlap = self._shared_overlap(x)
        h, x, base = self._pre_moe(x, batch, seq, segment_ids, not overlap)
        return self._moe(h, x, base, dp_group, logit_bias, overlap)


class Transformer(nn.Module):
    """Grug decoder (megagpt-speedrun/model.py:691-838; tiny-stories/model.py:138-226)."""

    def __init__(self, cfg: GrugModelConfig, local_experts=None, layers: range | None = None,
                 with_embed: bool = True, with_head: bool = True, tp=None):
        super().__init__()
        self.cfg = cfg
        d, de, v = cfg.hidden_dim, cfg.inferred_embed_dim, cfg.vocab_size
        self.layer_ids = list(layers) if layers is not None else list(range(cfg.num_layers))
        self.with_embed, self.with_head = with_embed, with_head
        if with_embed:
            self.token_embed = nn.Parameter(torch.empty(v, de))
            self.embed_up = nn.Parameter(torch.empty(d, de)) if cfg.is_factorized_embed else None
            self.embed_norm = NormPair(cfg) if cfg.is_moe else None
            ng = cfg.ngram
            self.ngram_table = (nn.Parameter(torch.empty(len(ng.orders), ng.hash_buckets, ng.rank))
                                if ng is not None else None)
            self.ngram_proj = nn.Parameter(torch.empty(d, ng.rank)) if ng is not None else None
        self.tp = tp
        self.blocks = nn.ModuleList([Block(cfg, i, local_experts, tp) for i in self.layer_ids])
        if with_head:
            self.final_norm = NormPair(cfg)
            self.head_down = nn.Parameter(torch.empty(de, d)) if cfg.is_factorized_embed else None
            self.output_proj = None if cfg.tie_embeddings else nn.Parameter(torch.empty(v, de))

    def global_name(self, name: str) -> str:
        """Parameter name in the full model: a pipeline stage's ``blocks.<j>`` is layer
        ``layer_ids[j]``, so seeds and checkpoint paths agree with the unsplit model."""
        if name.startswith("blocks."):
            j, rest = name[len("blocks."):].split(".", 1)
            return f"blocks.{self.layer_ids[int(j)]}.{rest}"
        return name

    # ------------------------------------------------------------------------------ init
    def init_weights(self, seed: int = 0):
        """Truncated-normal init with std ``initializer_std``; norms at 1, gates/biases at 0."""
        gen = torch.Generator(device="cpu").manual_seed(seed)
        std = self.cfg.initializer_std
        for name, p in self.named_parameters():
            leaf = name.rsplit(".", 1)[-1]
            if leaf == "weight":
                p.data.fill_(1.0)
            elif leaf in ("attn_gate", "router_bias"):
                p.data.zero_()
            elif leaf == "router_threshold":
                p.data.fill_(-4.0)
            else:
                cpu = torch.empty(p.shape, dtype=torch.float32)
                trunc_normal_(cpu, std, gen)
                p.data.copy_(cpu)
        return self

    # ---------------------------------------------------------------------------- forward
    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        x = ops.embed(tokens.reshape(-1), self.token_embed)
        if self.embed_up is not None:
            x = ops.linear(x, self.embed_up)
        if self.ngram_table is not None:  # hashed n-gram capacity added to the token embedding
            ng = self.cfg.ngram
            z = ops.ngram_embed(tokens.reshape(tokens.shape[0], -1), self.ngram_table, ng.orders, ng.num_hashes)
            x = ops.linear(z, self.ngram_proj, residual=x)
        if self.embed_norm is not None:
            x = self.embed_norm(x)
        return x

    def body(self, x, batch: int, seq: int, segment_ids=None, dp_group=None):
        stats = []
        for blk in self.blocks:
            x, st = blk(x, batch, seq, segment_ids, dp_group)
            if st is not None:
                stats.append(st)
        return x, stats

    def head_input(self, x):
        x = self.final_norm(x)
        if self.head_down is not None:
            x = ops.linear(x, self.head_down)
        return x

    def head_weight(self):
        return self.token_embed if self.output_proj is None else self.output_proj

    def forward(self, tokens, segment_ids=None, dp_group=None):
        b, s = tokens.shape
        x = self.embed(tokens)
        x, stats = self.body(x, b, s, None if segment_ids is None else segment_ids.reshape(-1), dp_group)
        return self.head_input(x), stats

    def logits(self, tokens, segment_ids=None):
        h, _ = self.forward(tokens, segment_ids)
        return h.float() @ self.head_weight().float().t()

    def next_token_loss(self, tokens, loss_weight=None, segment_ids=None, *, z_loss_weight: float = 0.0,
                        dp_group=None):
        """CE + router z-loss + sparsity penalty (+ LBL if ``aux_loss_coef``)
        (megagpt-speedrun/model.py:797-838). Returns ``(loss, metrics)``."""
        b, s = tokens.shape
        h, stats = self.forward(tokens, segment_ids, dp_group)
        labels = torch.cat([tokens[:, 1:], torch.zeros_like(tokens[:, :1])], dim=1).reshape(-1)
        if loss_weight is None:
            loss_weight = default_loss_weight(b, s, tokens.device)
        ce = ops.cross_entropy(h, self.head_weight(), labels, loss_weight.reshape(-1).float(),
                               z_weight=z_loss_weight)
        return combine_losses(self.cfg, ce, stats)


def default_loss_weight(b: int, s: int, device) -> torch.Tensor:
    w = torch.ones(b, s, device=device)
    w[:, -1] = 0.0
    return w


def combine_losses(cfg: GrugModelConfig, ce: torch.Tensor, stats: list[RouterStats]):
    metrics: dict[str, torch.Tensor] = {"train/cross_entropy_loss": ce.detach()}
    loss = ce
    if stats:
        n = len(stats)
        zl = torch.stack([s.z_loss for s in stats])
        lbl = torch.stack([s.lbl for s in stats])
        sp = torch.stack([s.sparsity for s in stats])
        aux = cfg.router_z_loss_coef * zl.sum() / n + cfg.sparsity_loss_coef * sp.mean()
        if cfg.aux_loss_coef:
            aux = aux + cfg.aux_loss_coef * lbl.mean()
        loss = ce + aux
        ent = torch.stack([s.entropy for s in stats]).detach()
        metrics.update({
            "train/router/router_z_loss": zl.detach().mean(),
            "train/router/load_balancing_loss": lbl.detach().mean(),
            "train/router/routing_entropy_mean": ent.mean(),
            "routing_entropy_per_layer": ent,
            "train/router/sparsity/realized_active_frac": torch.stack([s.realized_active_frac for s in stats]).detach().mean(),
            "train/router/sparsity/expected_active_frac": torch.stack([s.expected_active_frac for s in stats]).detach().mean(),
            "train/router/sparsity/threshold_mean": torch.stack([s.threshold for s in stats]).detach().float().mean(),
            "train/router/aux_loss_weighted": aux.detach(),
            "routing_counts_per_layer": torch.stack([s.counts for s in stats]).detach(),
        })
        if all(s.beta is not None for s in stats):
            metrics["qb_beta_per_layer"] = torch.stack([s.beta for s in stats]).detach()
    metrics["train/loss"] = loss.detach()
    return loss, metrics


def apply_qb_betas(model: Transformer, betas: torch.Tensor) -> None:
    """router_bias = -beta - mean(-beta), per MoE layer (megagpt-speedrun/train.py:320-332)."""
    i = 0
    with torch.no_grad():
        for blk in model.blocks:
            if isinstance(blk.mlp, MoEMLP):
                nb = -betas[i].float()
                nb = nb - nb.mean()
                blk.mlp.router_bias.copy_(nb.to(blk.mlp.router_bias.dtype))
                i += 1


def _seed_for(seed: int, name: str, sub: int = -1) -> int:
    import zlib

    return zlib.crc32(f"{seed}/{name}/{sub}".encode()) & 0x7FFFFFFF


def init_store_weights(store, cfg: GrugModelConfig, seed: int = 0, model: Transformer | None = None) -> None:
    """Initialise a model's flat parameter store in place on its device: truncated normal(-3, 3) *
    ``initializer_std`` for weight matrices, ones for norm scales, zeros for the attention gate and
    router bias, -4 for the adaptive threshold (megagpt-speedrun/model.py:234-253,488-519,841-842).

    Every parameter draws from its own generator seeded by (seed, name); routed-expert weights draw
    one generator per *global* expert id, so an expert-parallel shard holds exactly the experts the
    same model would have on one GPU."""
    std = cfg.initializer_std
    ranges = {}
    gname = model.global_name if model is not None and hasattr(model, "global_name") else (lambda n: n)
    mods = dict(model.named_modules()) if model is not None else {}

    def tp_module(name):
        m = mods.get(name.rsplit(".", 1)[0])
        tp = getattr(m, "tp", None)
        leaf = name.rsplit(".", 1)[-1]
        if tp is not None and tp.size > 1 and leaf in getattr(m, "tp_sharded_params", ()):
            return m, tp
        return None, None
    if model is not None:
        for mname, mod in model.named_modules():
            if isinstance(mod, MoEMLP):
                ranges[mname] = mod.expert_range
    with torch.no_grad():
        for info in store.infos:
            v = store.master_view(info)
            leaf = info.name.rsplit(".", 1)[-1]
            if leaf == "weight":
                v.fill_(1.0)
            elif leaf in ("attn_gate", "router_bias", "film_scale", "film_shift", "depth_bias", "halt_head"):
                v.zero_()
            elif leaf == "router_threshold":
                v.fill_(-4.0)
            elif leaf == "ngram_table":
                gen = torch.Generator(device=store.device).manual_seed(_seed_for(seed, gname(info.name)))
                trunc_normal_(v, std * cfg.ngram.ratio, gen)
            elif info.ndim == 3:
                lo = ranges.get(info.name.rsplit(".", 1)[0], (0, info.shape[0]))[0]
                for j in range(info.shape[0]):
                    gen = torch.Generator(device=store.device).manual_seed(_seed_for(seed, gname(info.name), lo + j))
                    trunc_normal_(v[j], std, gen)
            else:
                gen = torch.Generator(device=store.device).manual_seed(_seed_for(seed, gname(info.name)))
                m, tp = tp_module(info.name)
                if m is not None:  # tensor-parallel shard: slice of the full-size draw
                    from ..parallel.tp import full_shape, shard

                    full = torch.empty(full_shape(leaf, tuple(v.shape), m, tp), device=store.device)
                    trunc_normal_(full, std, gen)
                    v.copy_(shard(leaf, full, m, tp))
                else:
                    trunc_normal_(v, std, gen)
    store.sync_compute()
