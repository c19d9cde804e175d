"""Configuration dataclasses.

Field names follow the reference's frozen dataclasses so that a reference user finds the
same knobs:

* ``GrugModelConfig``   -- megagpt-speedrun/model.py:115-225 (MoE) and tiny-stories/model.py:22-55 (dense)
* ``GrugTrainerConfig`` -- megagpt-speedrun/train.py:56-77
* ``GrugEvalConfig``    -- megagpt-speedrun/train.py:80-90
* ``GrugRunConfig``     -- megagpt-speedrun/train.py:93-107
* ``CheckpointerConfig``-- levanter CheckpointerConfig as used at megagpt-speedrun/launch.py:152-165

Configs are plain frozen dataclasses; ``to_dict``/``from_dict`` give a JSON/YAML round trip
and ``apply_overrides`` implements ``--dotted.key=value`` command-line overrides.
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Any, Literal

RematMode = Literal["recompute_all", "save_moe", "none"]


@dataclass(frozen=True)
class RotaryConfig:
    """Rotary position embedding (levanter ``RotaryConfig`` default: theta 10000, no scaling).

    ``llama3_scaling`` reproduces the Llama-3 frequency scaling used by the Qwen3/Delphi patch
    (tunix-delphi-rl/models/delphi_patch.py:47-159)."""

    theta: float = 10000.0
    llama3_scaling: bool = False
    scaling_factor: float = 8.0
    low_freq_factor: float = 1.0
    high_freq_factor: float = 4.0
    original_max_position: int = 8192


@dataclass(frozen=True)
class NgramEmbedConfig:
    """Hashed multi-gram input embedding (Over-Encoding; tokenization/soak_config.py:15-29): one
    ``[hash_buckets, rank]`` table per n-gram order, ``num_hashes`` hash functions each, looked-up rows
    averaged, projected ``rank -> hidden`` and added to the token embedding. ``ratio`` scales the
    table init relative to the model's initializer std."""

    orders: tuple[int, ...] = (2, 3, 4)
    num_hashes: int = 2
    hash_buckets: int = 4_000_037
    rank: int = 128
    combine: Literal["mean"] = "mean"
    ratio: float = 0.25


@dataclass(frozen=True)
class GrugModelConfig:
    """Hyperparameters for the grug transformer (dense when ``num_experts == 0``).

    The MoE fields mirror megagpt-speedrun/model.py:115-225. Dense-only options
    (``mlp_activation``, ``glu``) cover the tiny-stories ReLU MLP (tiny-stories/model.py:104-108)
    and a SwiGLU dense MLP. ``aux_loss_coef`` adds the load-balancing loss to the objective
    (the reference computes it only as a metric, megagpt-speedrun/model.py:385-387).
    """

    vocab_size: int = 128256
    hidden_dim: int = 2048
    embed_dim: int | None = None
    intermediate_dim: int = 5632
    shared_expert_intermediate_dim: int = 5632
    num_experts: int = 8
    num_experts_per_token: int = 2
    adaptive_routing: bool = False
    min_experts_per_token: int = 0
    sparsity_loss_coef: float = 0.0
    sparsity_temp: float = 1.0
    num_layers: int = 24
    num_heads: int = 16
    num_kv_heads: int = 16
    head_dim: int | None = None
    max_seq_len: int = 4096
    sliding_window: int = 4096
    global_attn_every: int = 4
    local_window: int = 0
    layer_norm_eps: float = 1e-5
    initializer_std: float = 0.02
    qk_mult: float = 1.0
    router_z_loss_coef: float = 0.001
    aux_loss_coef: float = 0.0
    capacity_factor: float = 1.0
    # Accepted for config compatibility and ignored: this framework has one attention kernel, one
    # MoE path and one (exact) QB-beta selection, so there is nothing to choose between.
    attention_implementation: str | None = None
    moe_implementation: str | None = None
    fast_qb_beta: bool = False
    # Activation recompute per block: "none" keeps every activation; "recompute_all" keeps only each
    # block's input and recomputes the block in backward; "save_moe" keeps the routed-expert MoE's
    # activations and recomputes the rest of the block (norms, attention, shared expert).
    remat_mode: RematMode = "none"
    qb_balancing: bool = True
    # Architecture switches. The megagpt grug MoE has all of them on; the tiny dense template
    # has GatedNorm/QK-norm/XSA/head-gate off and a ReLU MLP.
    gated_norm: bool = True
    gated_norm_rank: int = 128
    qk_norm: bool = True
    xsa: bool = True
    head_gate: bool = True
    mlp_activation: Literal["silu", "relu", "gelu"] = "silu"
    glu: bool = True
    tie_embeddings: bool = False
    rope: RotaryConfig = field(default_factory=RotaryConfig)
    ngram: NgramEmbedConfig | None = None

    def __post_init__(self) -> None:
        _ = self.inferred_head_dim
        if self.remat_mode not in ("none", "recompute_all", "save_moe"):
            raise ValueError(f"remat_mode must be none, recompute_all or save_moe, got {self.remat_mode!r}")
        if self.num_heads % self.num_kv_heads != 0:
            raise ValueError("num_heads must be divisible by num_kv_heads for grouped-query attention")
        if self.vocab_size <= 0:
            raise ValueError("vocab_size must be positive")
        if self.max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if self.num_experts < 0:
            raise ValueError("num_experts must be non-negative")
        if self.num_experts > 0:
            if self.num_experts_per_token <= 0:
                raise ValueError("num_experts_per_token must be positive")
            if self.num_experts_per_token > self.num_experts:
                raise ValueError("num_experts_per_token must be <= num_experts")
            if self.min_experts_per_token < 0:
                raise ValueError("min_experts_per_token must be non-negative")
            if self.min_experts_per_token > self.num_experts_per_token:
                raise ValueError("min_experts_per_token must be <= num_experts_per_token (the K_max capacity)")
        if self.shared_expert_intermediate_dim < 0:
            raise ValueError("shared_expert_intermediate_dim must be non-negative")
        if self.glu:
            # gate/up weights are stored interleaved in 128-row blocks (SwiGLU in the GEMM epilogue)
            for name in ("intermediate_dim", "shared_expert_intermediate_dim"):
                v = getattr(self, name)
                if v % 128:
                    raise ValueError(f"{name}={v} must be a multiple of 128 for a GLU MLP")

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def inferred_embed_dim(self) -> int:
        return self.embed_dim if self.embed_dim is not None else self.hidden_dim

    @property
    def is_factorized_embed(self) -> bool:
        return self.inferred_embed_dim != self.hidden_dim

    @property
    def inferred_head_dim(self) -> int:
        if self.head_dim is not None:
            return self.head_dim
        if self.hidden_dim % self.num_heads != 0:
            raise ValueError(
                f"hidden_dim={self.hidden_dim} is not divisible by num_heads={self.num_heads}; set head_dim explicitly"
            )
        return self.hidden_dim // self.num_heads

    def layer_window(self, layer: int) -> int:
        """Attention window of ``layer`` (0 = unbounded causal).

        Every ``global_attn_every``-th layer is global (window ``sliding_window``); the others use
        ``local_window`` or ``sliding_window // 2`` (megagpt-speedrun/model.py:108-112,756-768).
        A window >= ``max_seq_len`` is reported as 0 (plain causal)."""
        g = max(1, self.global_attn_every)
        if layer % g == g - 1:
            w = self.sliding_window
        else:
            w = self.local_window if self.local_window > 0 else self.sliding_window // 2
        return 0 if w >= self.max_seq_len else w

    def param_count(self) -> dict[str, int]:
        """Total and active parameter counts (embeddings included)."""
        d, h = self.hidden_dim, self.inferred_head_dim
        de = self.inferred_embed_dim
        attn = d * self.num_heads * h * 2 + d * self.num_kv_heads * h * 2
        if self.head_gate:
            attn += d * self.num_heads
        gn = 2 * d * self.gated_norm_rank if self.gated_norm else 0
        per_layer = attn + 2 * d + 2 * gn
        active_layer = per_layer
        if self.is_moe:
            e_params = self.num_experts * 3 * d * self.intermediate_dim
            per_layer += e_params + d * self.num_experts
            active_layer += self.num_experts_per_token * 3 * d * self.intermediate_dim + d * self.num_experts
            if self.shared_expert_intermediate_dim:
                sh = 3 * d * self.shared_expert_intermediate_dim
                per_layer += sh
                active_layer += sh
        else:
            mlp = (3 if self.glu else 2) * d * self.intermediate_dim
            per_layer += mlp
            active_layer += mlp
        emb = self.vocab_size * de
        head = 0 if self.tie_embeddings else self.vocab_size * de
        fact = 2 * de * d if self.is_factorized_embed else 0
        extra = emb + head + fact + d + gn * 2
        return {
            "total": self.num_layers * per_layer + extra,
            "active": self.num_layers * active_layer + extra,
        }


@dataclass(frozen=True)
class CheckpointerConfig:
    """Checkpoint policy (levanter CheckpointerConfig fields, megagpt-speedrun/launch.py:152-165).

    ``save_interval_s`` is the wall-clock spacing of rolling temporary checkpoints (reference
    default 30 min); ``keep`` lists ``{"every": N}`` policies for permanent ones."""

    base_path: str = "checkpoints"
    temporary_base_path: str | None = None
    append_run_id_to_base_path: bool = False
    save_interval_s: float = 30 * 60
    keep_last_temporary_checkpoints: int = 2
    keep: tuple[dict[str, int], ...] | None = None
    save_final: bool = True


@dataclass(frozen=True)
class TrainerConfig:
    """The subset of levanter ``TrainerConfig`` the grug loop reads."""

    id: str | None = None
    seed: int = 0
    num_train_steps: int = 1000
    train_batch_size: int = 8
    per_device_parallelism: int = -1  # microbatch size in sequences per rank; -1 = whole local batch
    mp: str = "params=float32,compute=bfloat16,output=bfloat16"
    log_dir: str = "logs"
    checkpointer: CheckpointerConfig = field(default_factory=CheckpointerConfig)
    initialize_from: str | None = None
    load_checkpoint_path: str | None = None
    allow_partial_checkpoint: bool = False
    profiler: bool = False
    profiler_start_step: int = 5
    profiler_num_steps: int = 5
    watchdog_timeout_s: float = 0.0
    watch_every: int = 0  # gradient / parameter norms every N steps (0: off)
    watch_per_param: bool = False
    watch_hist_bins: int = 0


@dataclass(frozen=True)
class GrugTrainerConfig:
    """Trainer settings (megagpt-speedrun/train.py:56-77)."""

    trainer: TrainerConfig = field(default_factory=TrainerConfig)
    data_seed: int | None = None
    log_every: int = 1
    ema_beta: float | None = None
    z_loss_weight: float = 0.0
    expert_axis_size: int = 1
    replica_axis_size: int | None = None
    model_axis_size: int = 1
    pipeline_axis_size: int = 1


@dataclass(frozen=True)
class GrugEvalConfig:
    eval_batch_size: int = 512
    steps_per_eval: int | None = 1000
    max_eval_batches: int | None = None
    prefix: str = "eval"
    eval_current: bool = True
    eval_ema: bool = True
    compute_bpb: bool = True


@dataclass(frozen=True)
class DataConfig:
    """Data source. ``synthetic`` reproduces megagpt-speedrun/synth_data.py:25-70; ``cache``
    reads a token cache written by the tokenize step; ``mixture`` weights several caches; ``remote``
    is the named object-store mixture ``mix`` (``data.remote.MIXES``), mirrored under ``cache_dir``
    when the dataset is built (so a launch config can name it without touching the network)."""

    source: Literal["synthetic", "uniform", "cache", "mixture", "remote"] = "synthetic"
    seq_len: int = 4096
    cache_dir: str | None = None
    components: tuple[tuple[str, str, float], ...] = ()  # (name, cache_dir, weight)
    doc_len: int = 1024
    seed: int = 0
    prefetch: int = 4
    mix: str = ""


@dataclass(frozen=True)
class GrugRunConfig:
    """Top-level run config (megagpt-speedrun/train.py:93-107)."""

    model: GrugModelConfig = field(default_factory=GrugModelConfig)
    data: DataConfig = field(default_factory=DataConfig)
    optimizer: Any = None
    trainer: GrugTrainerConfig = field(default_factory=GrugTrainerConfig)
    eval: GrugEvalConfig | None = field(default_factory=GrugEvalConfig)
    k_schedule: tuple[tuple[int, int], ...] | None = None
    output_path: str = "out"


# ----------------------------------------------------------------------------- (de)serialisation


def to_dict(cfg: Any) -> Any:
    if dataclasses.is_dataclass(cfg) and not isinstance(cfg, type):
        out = {f.name: to_dict(getattr(cfg, f.name)) for f in dataclasses.fields(cfg)}
        out["__type__"] = type(cfg).__name__
        return out
    if isinstance(cfg, (list, tuple)):
        return [to_dict(x) for x in cfg]
    if isinstance(cfg, dict):
        return {k: to_dict(v) for k, v in cfg.items()}
    return cfg


def _registry() -> dict[str, type]:
    from . import optim  # noqa: F401  (registers optimizer configs)
    from .optim.base import OPTIMIZER_REGISTRY

    reg = {
        c.__name__: c
        for c in (
            RotaryConfig, NgramEmbedConfig, GrugModelConfig, CheckpointerConfig, TrainerConfig, GrugTrainerConfig,
            GrugEvalConfig, DataConfig, GrugRunConfig,
        )
    }
    for c in OPTIMIZER_REGISTRY.values():
        reg[c.__name__] = c
    return reg


def from_dict(d: Any) -> Any:
    if isinstance(d, dict) and "__type__" in d:
        cls = _registry()[d["__type__"]]
        kwargs = {}
        names = {f.name: f for f in dataclasses.fields(cls)}
        for k, v in d.items():
            if k == "__type__" or k not in names:
                continue
            kwargs[k] = from_dict(v)
            if isinstance(kwargs[k], list):
                kwargs[k] = _tuplify(kwargs[k])
        return cls(**kwargs)
    if isinstance(d, list):
        return [from_dict(x) for x in d]
    return d


def _tuplify(x: Any) -> Any:
    if isinstance(x, list):
        return tuple(_tuplify(v) for v in x)
    return x


def dumps(cfg: Any) -> str:
    return json.dumps(to_dict(cfg), indent=2, sort_keys=True, default=str)


def loads(s: str) -> Any:
    return from_dict(json.loads(s))


def _coerce(value: str, current: Any) -> Any:
    if isinstance(current, bool):
        return value.lower() in ("1", "true", "yes", "on")
    if isinstance(current, int) and not isinstance(current, bool):
        return int(value)
    if isinstance(current, float):
        return float(value)
    if current is None:
        for conv in (int, float):
            try:
                return conv(value)
            except ValueError:
                pass
        if value.lower() in ("none", "null"):
            return None
        if value.lower() in ("true", "false"):
            return value.lower() == "true"
        return value
    if isinstance(current, (tuple, list)):
        return tuple(json.loads(value))
    return value


def apply_overrides(cfg: Any, overrides: dict[str, str]) -> Any:
    """Apply ``{"model.hidden_dim": "768", ...}`` to a nested frozen dataclass."""
    for key, value in overrides.items():
        cfg = _set_path(cfg, key.split("."), value)
    return cfg


def _set_path(obj: Any, path: list[str], value: str) -> Any:
    head, rest = path[0], path[1:]
    if not dataclasses.is_dataclass(obj):
        raise KeyError(f"cannot set {'.'.join(path)} on {type(obj).__name__}")
    current = getattr(obj, head)
    new = _set_path(current, rest, value) if rest else _coerce(value, current)
    return dataclasses.replace(obj, **{head: new})


def parse_cli_overrides(argv: list[str]) -> tuple[dict[str, str], list[str]]:
    """Split ``--a.b=c`` / ``--a.b c`` dotted overrides from the other arguments."""
    overrides: dict[str, str] = {}
    rest: list[str] = []
    i = 0
    while i < len(argv):
        a = argv[i]
        if a.startswith("--") and "." in a.split("=")[0]:
            if "=" in a:
                k, v = a[2:].split("=", 1)
            else:
                k, v = a[2:], argv[i + 1]
                i += 1
            overrides[k] = v
        else:
            rest.append(a)
        i += 1
    return overrides, rest
