"""Named base models: aliases, architecture checks of local checkpoints, random-init by name."""

import json
import os
from dataclasses import replace

import pytest
import torch

from marin_experiments_b200.models import registry as R


def test_names_and_aliases():
    assert R.get_spec("Delphi-447M").name == "delphi" and R.get_spec("qwen3").name == "qwen3-1.7b-base"
    assert R.get_spec("delphi-2b").repo.endswith("1.9Bparams-24.7Btokens")
    with pytest.raises(KeyError, match="unknown model"):
        R.get_spec("gpt2")
    d = R.get_spec("delphi").config
    n = d.vocab_size * d.hidden_dim * 2 + d.num_layers * (
        d.hidden_dim * d.head_dim * (2 * d.num_heads + 2 * d.num_kv_heads) + 3 * d.hidden_dim * d.intermediate_dim)
    assert 4.3e8 < n < 4.7e8  # the 447M of the checkpoint's name
    q8 = R.get_spec("qwen3-8b").config
    n8 = q8.vocab_size * q8.hidden_dim * 2 + q8.num_layers * (
        q8.hidden_dim * q8.head_dim * (2 * q8.num_heads + 2 * q8.num_kv_heads) + 3 * q8.hidden_dim * q8.intermediate_dim)
    assert 7.9e9 < n8 < 8.4e9
    with pytest.raises(ValueError, match="no registered architecture"):
        R.build("delphi-1.9b")


def test_checkpoint_checks_and_load(tmp_path, monkeypatch):
    from marin_experiments_b200.models.qwen3_export import export_hf

    small = replace(R.get_spec("delphi").config, vocab_size=512, hidden_dim=128, intermediate_dim=256, num_layers=2,
                    num_heads=2, num_kv_heads=2, head_dim=64, max_seq_len=128)
    monkeypatch.setitem(R.REGISTRY, "tiny", R.ModelSpec("tiny", "local/tiny", small))
    m = R.build("tiny", seed=1)
    d = export_hf(m, str(tmp_path / "ck"), dtype=torch.float32)
    got = R.load("tiny", d, dtype=torch.float32)
    x = torch.randint(0, 512, (1, 16))
    assert torch.allclose(got.forward_logits(x), m.forward_logits(x), atol=1e-4)
    with pytest.raises(ValueError, match="does not hold delphi"):
        R.check_checkpoint("delphi", d)
    cfg = json.load(open(os.path.join(d, "config.json")))
    cfg.pop("rope_scaling")
    json.dump(cfg, open(os.path.join(d, "config.json"), "w"))
    with pytest.raises(ValueError, match="Llama-3 RoPE scaling"):
        R.check_checkpoint("tiny", d)


def test_llama3_rope_matches_transformers():
    """The Llama-3 RoPE frequency scaling (Delphi's rope setup) against transformers' own implementation."""
    import warnings

    from transformers import Qwen3Config as HFQwen3Config
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    from marin_experiments_b200.ops import reference as OR

    spec = R.get_spec("delphi").config
    hf = HFQwen3Config(hidden_size=spec.hidden_dim, num_attention_heads=spec.num_heads, head_dim=spec.head_dim,
                       rope_theta=spec.rope_theta, rope_scaling=dict(spec.rope_scaling), max_position_embeddings=16384)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        want, _ = ROPE_INIT_FUNCTIONS["llama3"](hf, "cpu")
    base = 1.0 / (spec.rope_theta ** (torch.arange(0, spec.head_dim, 2, dtype=torch.float64) / spec.head_dim))
    got = OR.llama3_scale_inv_freq(base, **spec.llama3())
    assert torch.allclose(got.double(), want.double(), rtol=1e-6, atol=0)
    assert not torch.allclose(base, want.double(), rtol=1e-3)  # the scaling changes most components
