"""megagpt-speedrun launcher: environment-variable arms -> one executor step
(megagpt-speedrun/launch.py:203-573).

The model and AdamH hyperparameters come from the compute-scaling heuristic (``SP_HIDDEN``,
``SP_EXPERTS``, ``SP_TOPK``, ``SP_TOKENS`` or ``SP_BUDGET``, ``SP_FIT_BATCH``), with overrides for the
throughput levers (``SP_EMBED``, ``SP_SEQ``, ``SP_INTERMEDIATE``, ``SP_GLOBAL_EVERY``,
``SP_LOCAL_WINDOW``, ``SP_REMAT``, ``SP_MOE_IMPL``, ``SP_ATTN``, ``SP_FAST_QB``), the schedule
(``SP_SCHEDULE``, ``SP_WARMUP``, ``SP_DECAY``, ``SP_MIN_LR``, ``SP_REWARMUP``), the mesh (``SP_EP``,
``SP_TP``, ``SP_REPLICA``), adaptive sparsity (``SPARSITY_MODE=adaptive``, ``SP_MIN_K``, ``SP_COEF``,
``SP_TEMP``), the k-curriculum (``SP_CURRICULUM="k:frac,..."``), weights-only init (``SP_INIT_FROM``),
raw overrides (``SP_BATCH``, ``SP_STEPS``), data (``SP_DATA``: ``synthetic``, a token cache path, or a
named object-store mixture -- ``datakit`` / ``nemotron``, ``nemotron-full``, ``sft`` -- mirrored under
``MXK_DATA_ROOT`` from ``MXK_CORPUS_PREFIX`` when training starts;
``SP_SYNTH_DATA=1`` forces synthetic), eval (``SP_EVAL``, ``SP_EVAL_ONLY``, ``SP_EVAL_BS``,
``SP_EVAL_MAXB``) and ``SP_TAG``. ``SP_PP_MODE=async|sync`` runs the pipeline-parallel entry points
instead. The ``[arm]`` line printed per launch is the one the sweep monitor parses.
"""

from __future__ import annotations

import dataclasses
import os
import sys

from ..config import DataConfig, GrugEvalConfig, GrugTrainerConfig
from ..executor import ExecutorStep, executor_main, this_output_path, versioned
from ..optim.heuristic import MoeAdamHHeuristic, build_from_heuristic
from ..train.curriculum import parse_curriculum
from ..utils.flops import compute_flops_per_token
from .common import GrugLaunchConfig, run_inline


def _env(env, key: str, default: str) -> str:
    v = env.get(key, "")
    return v if v else default


def make_launch(env=None) -> tuple[GrugLaunchConfig, str]:
    env = os.environ if env is None else env
    mode = _env(env, "SPARSITY_MODE", "fixed")
    hidden = int(_env(env, "SP_HIDDEN", "512"))
    num_experts = int(_env(env, "SP_EXPERTS", "1024"))
    top_k = int(_env(env, "SP_TOPK", "4"))
    min_k = int(_env(env, "SP_MIN_K", "0"))
    coef = float(_env(env, "SP_COEF", "0.0"))
    temp = float(_env(env, "SP_TEMP", "1.0"))
    ref_top_k = int(_env(env, "SP_REF_TOPK", "4"))
    target_tokens = _env(env, "SP_TOKENS", "")
    fit_batch = _env(env, "SP_FIT_BATCH", "")
    seed = int(_env(env, "SP_SEED", "0"))
    embed = _env(env, "SP_EMBED", "")
    embed_dim = int(embed) if embed else None
    seq = int(_env(env, "SP_SEQ", "4096"))
    ep = int(_env(env, "SP_EP", "1"))
    tp = int(_env(env, "SP_TP", "1"))
    rep = _env(env, "SP_REPLICA", "")
    remat = _env(env, "SP_REMAT", "recompute_all")
    moe_impl = _env(env, "SP_MOE_IMPL", "") or None
    log_every = int(_env(env, "SP_LOG_EVERY", "1"))
    fast_qb = _env(env, "SP_FAST_QB", "0") == "1"
    attn = _env(env, "SP_ATTN", "sm100_flash") or None
    inter = int(_env(env, "SP_INTERMEDIATE", "0"))
    global_every = int(_env(env, "SP_GLOBAL_EVERY", "0"))
    local_window = int(_env(env, "SP_LOCAL_WINDOW", "0"))
    curriculum = _env(env, "SP_CURRICULUM", "")
    if curriculum:
        mode = "fixed"
        top_k = int(curriculum.split(",")[0].split(":")[0])
    if mode not in ("fixed", "adaptive"):
        raise ValueError(f"SPARSITY_MODE must be 'fixed' or 'adaptive', got {mode!r}")
    adaptive = mode == "adaptive"
    h = MoeAdamHHeuristic()
    ref = h.build_model_config(hidden, seq_len=seq, num_experts=num_experts, num_experts_per_token=ref_top_k,
                               embed_dim=embed_dim)
    budget = 3.0 * compute_flops_per_token(ref) * float(target_tokens) if target_tokens else \
        float(_env(env, "SP_BUDGET", "1.7e18"))
    if fit_batch and not target_tokens:
        raise ValueError("SP_FIT_BATCH requires SP_TOKENS")
    _, opt, ref_batch, ref_steps = build_from_heuristic(
        budget=budget, hidden_dim=hidden, seq_len=seq, batch_size=int(fit_batch) if fit_batch else None,
        model_overrides=dict(num_experts=num_experts, num_experts_per_token=ref_top_k, embed_dim=embed_dim))
    sched = {}
    for key, field_, conv in (("SP_SCHEDULE", "lr_schedule", str), ("SP_WARMUP", "warmup", float),
                              ("SP_DECAY", "decay", float), ("SP_MIN_LR", "min_lr_ratio", float),
                              ("SP_REWARMUP", "rewarmup", float)):
        if env.get(key, "") != "":
            sched[field_] = conv(env[key])
    if sched:
        opt = dataclasses.replace(opt, **sched)
    model = h.build_model_config(hidden, seq_len=seq, num_experts=num_experts, num_experts_per_token=top_k,
                                 adaptive_routing=adaptive, min_experts_per_token=min_k,
                                 sparsity_loss_coef=coef if adaptive else 0.0, sparsity_temp=temp, embed_dim=embed_dim)
    over = dict(remat_mode=remat, moe_implementation=moe_impl, fast_qb_beta=fast_qb, attention_implementation=attn)
    if inter > 0:
        over["intermediate_dim"] = inter
    if global_every > 0:
        over["global_attn_every"] = global_every
    if local_window > 0:
        over["local_window"] = local_window
    model = dataclasses.replace(model, **over)
    batch = int(_env(env, "SP_BATCH", str(ref_batch)))
    steps = int(_env(env, "SP_STEPS", str(ref_steps)))
    k_schedule = parse_curriculum(curriculum, steps) if curriculum else None
    if curriculum:
        ks = [k for k, _ in k_schedule]
        arm = f"curric-d{hidden}-E{num_experts}-k{ks[0]}to{ks[-1]}"
    elif adaptive:
        arm = f"adapt-d{hidden}-E{num_experts}-k{top_k}-min{min_k}-c{coef:g}-t{temp:g}"
    else:
        arm = f"fixed-d{hidden}-E{num_experts}-k{top_k}"
    if inter > 0:
        arm += f"-I{inter}"
    if embed_dim is not None:
        arm += f"-de{embed_dim}"
    run_id = f"sparsity-{arm}-s{seed}-st{steps}"
    if env.get("SP_TAG"):
        run_id += f"-{env['SP_TAG']}"
    data_kind = _env(env, "SP_DATA", "synthetic")
    remote_mix = {"datakit": "nemotron", "datakit_eval": "nemotron", "nemotron": "nemotron",
                  "nemotron-full": "nemotron-full", "sft": "sft-chat", "sft-chat": "sft-chat"}.get(data_kind)
    if env.get("SP_SYNTH_DATA", "").strip().lower() in ("1", "true", "yes") or data_kind == "synthetic":
        data = DataConfig(source="synthetic", seed=seed)
    elif remote_mix:  # the reference's object-store mixtures, mirrored under MXK_DATA_ROOT at run time
        data = DataConfig(source="remote", mix=remote_mix, cache_dir=os.environ.get("MXK_DATA_ROOT", "data_cache"),
                          seed=seed)
    else:
        data = DataConfig(source="cache", cache_dir=data_kind, seed=seed)
    ev = None
    if env.get("SP_EVAL") == "1":
        maxb = env.get("SP_EVAL_MAXB", "")
        ev = GrugEvalConfig(eval_batch_size=int(_env(env, "SP_EVAL_BS", "16")), steps_per_eval=10 ** 9,
                            max_eval_batches=int(maxb) if maxb else None, eval_current=True, eval_ema=False)
    launch = GrugLaunchConfig(
        model=versioned(model), data=data, output_path=this_output_path(), run_id=run_id, steps=versioned(steps),
        batch_size=versioned(batch), seed=versioned(seed),
        mp=versioned("params=float32,compute=bfloat16,output=bfloat16"), optimizer=versioned(opt),
        grug_trainer=versioned(GrugTrainerConfig(z_loss_weight=1e-4, ema_beta=None, log_every=log_every,
                                                 expert_axis_size=ep, model_axis_size=tp,
                                                 replica_axis_size=int(rep) if rep else None)),
        k_schedule=k_schedule, init_from=env.get("SP_INIT_FROM") or None, eval=ev,
        eval_only=env.get("SP_EVAL_ONLY") == "1")
    arm_line = (f"[arm] {run_id}  mode={mode} D={hidden} d_e={model.inferred_embed_dim}"
                f"(factorized={model.is_factorized_embed}) seq={seq} E={num_experts} k={top_k} min_k={min_k} "
                f"coef={coef} nominal_active_frac={top_k / num_experts:.4%} batch={batch} steps={steps} "
                f"tokens={batch * steps * seq / 1e9:.1f}B layers={model.num_layers} I_expert={model.intermediate_dim} "
                f"mesh(EP={ep},TP={tp},replica={rep or None}) data={data_kind} budget={budget:g} remat={remat} "
                f"moe_impl={moe_impl} attn={attn} curriculum={k_schedule}")
    return launch, arm_line


def make_step(env=None) -> ExecutorStep:
    launch, arm = make_launch(env)
    print(arm, flush=True)
    return ExecutorStep(name=f"grug/sparsity/{launch.run_id}", fn=run_inline, config=launch)


def main(argv=None):
    if os.environ.get("SP_DIAG"):  # diagnostic side entries (ragged / ring / fit / attn)
        from ..benchmarks import diag

        diag.main(os.environ["SP_DIAG"])
        return None
    mode = os.environ.get("SP_PP_MODE", "")
    if mode in ("async", "sync"):
        from ..parallel import pipeline_entry

        (pipeline_entry.run_pp_async if mode == "async" else pipeline_entry.run_pp_sync)()
        return None
    return executor_main([make_step()], description="Grug MoE sparsity / speedrun launcher.", argv=argv)


if __name__ == "__main__":
    main(sys.argv[1:])
