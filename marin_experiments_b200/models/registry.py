"""Named base models for post-training (tunix-delphi-rl/models/registry.py,
openthoughts-agent/models/registry.py): a name (or alias) -> the Hugging Face repository, and,
where the architecture is public, its ``Qwen3Config``.

The config lets a user build a random-init model of the right shape by name (benchmarks, memory
fits, smoke runs on a machine with no network); ``load(name, model_dir)`` loads a local
checkpoint directory and checks that its ``config.json`` matches the registered architecture, so a
directory holding a different model fails loudly instead of training the wrong one. Specs without a
config take theirs from the checkpoint.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass

from .qwen3 import Qwen3Config

_LLAMA3_ROPE = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                "original_max_position_embeddings": 8192}


@dataclass(frozen=True)
class ModelSpec:
    name: str
    repo: str
    config: Qwen3Config | None = None
    note: str = ""


# Architectures are the published configurations of these checkpoints.
_SPECS = [
    ModelSpec("delphi", "marin-community/delphi-3e18-447Mparams-1.2Btokens",
              Qwen3Config(vocab_size=128256, hidden_dim=1024, intermediate_dim=4096, num_layers=11, num_heads=8,
                          num_kv_heads=8, head_dim=128, rope_theta=500000.0, rope_scaling=dict(_LLAMA3_ROPE),
                          norm_eps=1e-5, tie_embeddings=False, max_seq_len=4096),
              "447M base LM; Llama-3 RoPE scaling with theta 500000"),
    ModelSpec("delphi-1.9b", "marin-community/delphi-3e20-1.9Bparams-24.7Btokens", None,
              "the ~2B point of the same ladder, width 2048; config read from the checkpoint"),
    ModelSpec("qwen3-1.7b-base", "Qwen/Qwen3-1.7B-Base",
              Qwen3Config(vocab_size=151936, hidden_dim=2048, intermediate_dim=6144, num_layers=28, num_heads=16,
                          num_kv_heads=8, head_dim=128, rope_theta=1_000_000.0, norm_eps=1e-6, tie_embeddings=True,
                          max_seq_len=32768)),
    ModelSpec("qwen3-8b", "Qwen/Qwen3-8B",
              Qwen3Config(vocab_size=151936, hidden_dim=4096, intermediate_dim=12288, num_layers=36, num_heads=32,
                          num_kv_heads=8, head_dim=128, rope_theta=1_000_000.0, norm_eps=1e-6, tie_embeddings=False,
                          max_seq_len=40960), "chat model (ChatML), the terminal-agent recipe's start"),
    ModelSpec("qwen3-8b-base", "Qwen/Qwen3-8B-Base",
              Qwen3Config(vocab_size=151936, hidden_dim=4096, intermediate_dim=12288, num_layers=36, num_heads=32,
                          num_kv_heads=8, head_dim=128, rope_theta=1_000_000.0, norm_eps=1e-6, tie_embeddings=False,
                          max_seq_len=32768)),
]
_ALIASES = {"delphi-447m": "delphi", "delphi-2b": "delphi-1.9b", "delphi-1.9b-base": "delphi-1.9b",
            "qwen3": "qwen3-1.7b-base", "qwen3-1.7b": "qwen3-1.7b-base"}
REGISTRY = {s.name: s for s in _SPECS}


def get_spec(name: str) -> ModelSpec:
    key = name.strip().lower()
    key = _ALIASES.get(key, key)
    if key not in REGISTRY:
        raise KeyError(f"unknown model {name!r}; known: {sorted(REGISTRY) + sorted(_ALIASES)}")
    return REGISTRY[key]


def _arch(c: Qwen3Config) -> tuple:
    return (c.vocab_size, c.hidden_dim, c.intermediate_dim, c.num_layers, c.num_heads, c.num_kv_heads, c.head_dim,
            c.tie_embeddings)


def check_checkpoint(name: str, model_dir: str) -> Qwen3Config:
    """The checkpoint's config, after checking it against the registered architecture."""
    with open(os.path.join(model_dir, "config.json")) as f:
        got = Qwen3Config.from_hf(json.load(f))
    spec = get_spec(name)
    if spec.config is not None and _arch(got) != _arch(spec.config):
        raise ValueError(f"{model_dir} does not hold {spec.name} ({spec.repo}): architecture {_arch(got)} != "
                         f"{_arch(spec.config)} (vocab, hidden, intermediate, layers, heads, kv heads, head dim, tied)")
    if spec.config is not None and spec.config.rope_scaling and not got.rope_scaling:
        raise ValueError(f"{model_dir}: {spec.name} needs Llama-3 RoPE scaling; config.json has none")
    return got


def build(name: str, seed: int = 0, **overrides):
    """A random-init ``Qwen3Model`` of the registered architecture (``overrides`` change config fields,
    e.g. ``max_seq_len``)."""
    from dataclasses import replace

    from .qwen3 import Qwen3Model

    spec = get_spec(name)
    if spec.config is None:
        raise ValueError(f"{spec.name}: no registered architecture; load it from a checkpoint")
    return Qwen3Model(replace(spec.config, **overrides)).init_weights(seed)


def load(name: str, model_dir: str, device="cpu", dtype=None):
    """The checkpoint in ``model_dir`` (safetensors + config.json), checked against ``name``."""
    import torch

    from .qwen3 import load_hf

    check_checkpoint(name, model_dir)
    return load_hf(model_dir, device=device, dtype=dtype or torch.bfloat16)
