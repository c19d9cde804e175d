"""Export a ``Qwen3Model`` as a Hugging Face ``Qwen3ForCausalLM`` snapshot: ``config.json`` plus
``model.safetensors`` in HF parameter names and layouts (tunix-delphi-rl/serving/export_hf.py:54-269).
The block-interleaved gate/up rows are split back into ``gate_proj`` / ``up_proj``."""

from __future__ import annotations

import json
import os

import torch

from ..ops.layout import blocked_rows_to_gate_up
from .qwen3 import _HF_LAYER, Qwen3Model


def export_hf(model: Qwen3Model, out_dir: str, dtype=torch.bfloat16) -> str:
    from safetensors.torch import save_file

    os.makedirs(out_dir, exist_ok=True)
    c = model.cfg
    sd = {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.final_norm}
    if model.lm_head is not None:
        sd["lm_head.weight"] = model.lm_head
    for i, L in enumerate(model.layers):
        pre = f"model.layers.{i}."
        for hk, ours in _HF_LAYER.items():
            sd[pre + hk] = getattr(L, ours)
        g, u = blocked_rows_to_gate_up(L.w_gate_up.detach().float())
        sd[pre + "mlp.gate_proj.weight"] = g
        sd[pre + "mlp.up_proj.weight"] = u
    out = {k: v.detach().to("cpu", dtype).contiguous() for k, v in sd.items()}
    save_file(out, os.path.join(out_dir, "model.safetensors"))
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(c.to_hf(), f, indent=1)
    return out_dir
