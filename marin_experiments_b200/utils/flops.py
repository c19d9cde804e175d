"""FLOP accounting (megagpt-speedrun/train.py:225-250, megagpt-speedrun/perf_flop_breakdown.py:24-85).

All counts are forward FLOPs per token (2 x multiply-accumulates) unless the name says otherwise;
training = 3 x forward. Attention scores follow the analytic per-token convention of the reference's
breakdown: ``(2 S^2 H hd + 3 S^2 H + 2 S^2 H hd) / S`` (scores, softmax/mask, weighted values) for a
full S x S score matrix. GatedNorms (two D x r matmuls each, two per block plus embed and final) are
counted by ``fwd_components`` and omitted by ``lm_flops_per_token``, like the reference's split
between its analytic breakdown and the library count it logs.
"""

from __future__ import annotations


def fwd_components(cfg, k: int | None = None) -> dict[str, float]:
    """Forward FLOPs per token by component, for ``k`` active routed experts (default: the config's)."""
    k = cfg.num_experts_per_token if k is None else k
    d, e, l_ = cfg.hidden_dim, cfg.num_experts, cfg.num_layers
    h, kv, hd, s, v = cfg.num_heads, cfg.num_kv_heads, cfg.inferred_head_dim, cfg.max_seq_len, cfg.vocab_size
    de = cfg.inferred_embed_dim
    qkv = 2 * d * (h * hd + 2 * kv * hd)
    o = 2 * (h * hd) * d
    scores = (2 * s * s * h * hd + 3 * s * s * h + 2 * s * s * hd * h) / s
    router = 2 * d * e if e > 0 else 0
    mats = 3 if cfg.glu else 2
    routed = 2 * mats * d * cfg.intermediate_dim * k if e > 0 else 0
    dense_mlp = 0 if e > 0 else 2 * mats * d * cfg.intermediate_dim
    shared = 2 * mats * d * cfg.shared_expert_intermediate_dim if e > 0 else 0
    r = cfg.gated_norm_rank
    gn = 2 * (2 * d * r) if cfg.gated_norm else 0
    head = 2 * de * v + (2 * 2 * d * de if de != d else 0)  # factorized: embed_up + head_down
    comps = {
        "attn_proj_QKVO": l_ * (qkv + o),
        "attn_scores_AV": l_ * scores,
        "router_proj": l_ * router,
        "routed_experts": l_ * routed,
        "shared_expert": l_ * shared,
        "dense_mlp": l_ * dense_mlp,
        "gated_norms": l_ * 2 * gn + 2 * gn,
        "lm_head": head,
    }
    comps["attention"] = comps["attn_proj_QKVO"] + comps["attn_scores_AV"]
    comps["_total"] = sum(v for k_, v in comps.items() if k_ not in ("attention",))
    return comps


def lm_flops_per_token(cfg) -> float:
    """Forward FLOPs per token including the LM head, without GatedNorms."""
    c = fwd_components(cfg)
    return c["_total"] - c["gated_norms"]


def compute_flops_per_token(cfg) -> float:
    """Non-embedding forward FLOPs per token (excludes the LM head): the compute-budget unit of the
    scaling heuristic, ``C = 3 * compute_flops_per_token * tokens``."""
    return lm_flops_per_token(cfg) - 2 * cfg.hidden_dim * cfg.vocab_size


def training_flops_per_token(cfg, causal: bool = True) -> float:
    """Forward + backward FLOPs per token of everything the step computes (GatedNorms included).
    ``causal`` counts half of the score matrix, the work a causal flash-attention kernel does."""
    c = fwd_components(cfg)
    tot = c["_total"]
    if causal:
        tot -= c["attn_scores_AV"] / 2
    return 3.0 * tot


def flops_summary(cfg) -> dict[str, float]:
    f = lm_flops_per_token(cfg)
    return {"throughput/flops_per_token_analytic": f,
            "throughput/flops_per_example_analytic": 3 * f * cfg.max_seq_len}


def mfu(tokens_per_s: float, cfg, n_gpus: int, peak_flops: float = 2.25e15) -> float:
    return tokens_per_s * training_flops_per_token(cfg) / (n_gpus * peak_flops)
