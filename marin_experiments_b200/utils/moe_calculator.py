"""Browser calculator for MoE geometry: parameters, FLOPs per token, MFU and tokens x parameters.

The reference ships a browser page that restates its FLOP math for interactive geometry
exploration (megagpt-speedrun/moe_calculator.html). Here the formulas live once, in ``FORMULAS``, as
arithmetic expressions in the common subset of Python and JavaScript (numbers, names, ``+ - * /``,
parentheses, comparisons used as 0/1 factors). ``evaluate`` computes them in Python, and the tests
hold them equal to ``utils.flops`` and ``utils.perf_model.param_split``. ``render`` writes a
self-contained HTML page (no external scripts) whose JavaScript evaluates the same strings;
``moe_calculator.html`` beside this file is its output for the megagpt geometry:

    python -m marin_experiments_b200.utils.moe_calculator > marin_experiments_b200/utils/moe_calculator.html
"""

from __future__ import annotations

import html
import json

# (name, label, default): D hidden, DE embedding width (= D unless factorized), I routed-expert width
# (or dense MLP width when E = 0), SI shared-expert width, L layers, V vocabulary, E experts, K
# experts per token, H / KV query / key-value heads, HD head dim, S sequence, R GatedNorm rank, GN
# GatedNorms on (1/0), M matrices per MLP (3 GLU, 2 plain), TIE tied embeddings (1/0); run: TPS
# tokens/s of the whole job, GPUS, PEAK dense bf16 FLOP/s per GPU, HOURS of training.
INPUTS = [
    ("D", "hidden size", 1536), ("DE", "embedding width", 1536), ("I", "expert width", 768),
    ("SI", "shared-expert width", 3072), ("L", "layers", 24), ("V", "vocabulary", 128256),
    ("E", "experts", 64), ("K", "experts per token", 4), ("H", "query heads", 16), ("KV", "kv heads", 4),
    ("HD", "head dim", 96), ("S", "sequence length", 2048), ("R", "GatedNorm rank", 128),
    ("GN", "GatedNorms (1/0)", 1), ("M", "matrices per MLP (3 GLU / 2)", 3), ("TIE", "tied embeddings (1/0)", 0),
    ("TPS", "measured tokens/s (whole job)", 662754), ("GPUS", "GPUs", 8), ("PEAK", "peak FLOP/s per GPU", 2.25e15),
    ("HOURS", "training hours", 24),
]

# (name, label, expression); an expression may use the inputs and the names defined above it.
FORMULAS = [
    ("qkv", "QKV projection FLOPs / token / layer", "2 * D * (H * HD + 2 * KV * HD)"),
    ("o", "O projection FLOPs / token / layer", "2 * (H * HD) * D"),
    ("scores", "attention scores + AV FLOPs / token / layer (full S x S)",
     "(2 * S * S * H * HD + 3 * S * S * H + 2 * S * S * HD * H) / S"),
    ("f_attn_proj", "fwd: attention projections", "L * (qkv + o)"),
    ("f_attn_scores", "fwd: attention scores", "L * scores"),
    ("f_router", "fwd: router", "L * 2 * D * E * (E > 0)"),
    ("f_routed", "fwd: routed experts", "L * 2 * M * D * I * K * (E > 0)"),
    ("f_shared", "fwd: shared expert", "L * 2 * M * D * SI * (E > 0)"),
    ("f_dense", "fwd: dense MLP", "L * 2 * M * D * I * (E == 0)"),
    ("f_gated", "fwd: GatedNorms", "(L * 2 + 2) * (2 * (2 * D * R)) * GN"),
    ("f_head", "fwd: LM head (+ factorized embed up / head down)", "2 * DE * V + 2 * 2 * D * DE * (DE != D)"),
    ("fwd", "forward FLOPs / token",
     "f_attn_proj + f_attn_scores + f_router + f_routed + f_shared + f_dense + f_gated + f_head"),
    ("train", "training FLOPs / token (3 x forward, causal attention)", "3 * (fwd - f_attn_scores / 2)"),
    ("p_experts", "routed-expert parameters", "L * E * M * D * I * (E > 0)"),
    ("p_attn", "attention parameters (q, k, v, o, head gate)", "L * (D * HD * (2 * H + 2 * KV) + H * D)"),
    ("p_mlp", "shared-expert / dense MLP parameters", "L * M * D * (SI * (E > 0) + I * (E == 0))"),
    ("p_router", "router parameters", "L * D * E * (E > 0)"),
    ("p_embed", "embedding + output parameters", "V * DE * (2 - TIE)"),
    ("p_total", "total parameters", "p_experts + p_attn + p_mlp + p_router + p_embed"),
    ("p_active", "active parameters per token", "p_experts * K / (E + (E == 0)) + p_total - p_experts"),
    ("mfu", "MFU at the measured tokens/s", "TPS * train / (GPUS * PEAK)"),
    ("tokens", "tokens in the training hours", "TPS * 3600 * HOURS"),
    ("tok_x_total", "tokens x total parameters", "tokens * p_total"),
    ("tok_x_active", "tokens x active parameters", "tokens * p_active"),
    ("tok_per_expert", "routed tokens per expert over the run", "tokens * K / (E + (E == 0)) * (E > 0)"),
]


def inputs_from_config(cfg, **run) -> dict:
    v = {k: d for k, _, d in INPUTS}
    v.update(D=cfg.hidden_dim, DE=cfg.inferred_embed_dim, I=cfg.intermediate_dim,
             SI=cfg.shared_expert_intermediate_dim, L=cfg.num_layers, V=cfg.vocab_size, E=cfg.num_experts,
             K=cfg.num_experts_per_token, H=cfg.num_heads, KV=cfg.num_kv_heads, HD=cfg.inferred_head_dim,
             S=cfg.max_seq_len, R=cfg.gated_norm_rank, GN=1 if cfg.gated_norm else 0, M=3 if cfg.glu else 2,
             TIE=1 if cfg.tie_embeddings else 0)
    v.update(run)
    return v


def evaluate(values: dict) -> dict:
    """All formulas, in order, over ``values`` (the inputs); returns inputs and results."""
    env = dict(values)
    for name, _, expr in FORMULAS:
        env[name] = float(eval(expr, {"__builtins__": {}}, env))  # expressions are this module's constants
    return env


_PAGE = """<!doctype html>
<html lang="en"><head><meta charset="utf-8"><title>MoE geometry calculator</title>
<style>
body {{ font: 14px system-ui, sans-serif; margin: 24px; max-width: 1100px; }}
.grid {{ display: grid; grid-template-columns: repeat(4, 1fr); gap: 6px 16px; margin-bottom: 18px; }}
label {{ display: flex; justify-content: space-between; gap: 8px; }}
input {{ width: 9em; }}
table {{ border-collapse: collapse; }} td {{ padding: 2px 10px; border-bottom: 1px solid #ddd; }}
td.v {{ text-align: right; font-variant-numeric: tabular-nums; }}
</style></head><body>
<h2>MoE geometry calculator</h2>
<p>Parameters, FLOPs per token (forward = 2 x multiply-accumulates; training = 3 x forward with causal
attention), MFU and tokens x parameters. Formulas are those of the framework's FLOP accounting.</p>
<div class="grid" id="inputs"></div>
<table id="out"></table>
<script>
const INPUTS = {inputs};
const FORMULAS = {formulas};
function fmt(x) {{
  const a = Math.abs(x);
  if (a >= 1e15) return (x / 1e15).toFixed(3) + " P";
  if (a >= 1e12) return (x / 1e12).toFixed(3) + " T";
  if (a >= 1e9) return (x / 1e9).toFixed(3) + " G";
  if (a >= 1e6) return (x / 1e6).toFixed(3) + " M";
  if (a >= 1e3) return (x / 1e3).toFixed(3) + " K";
  return x.toPrecision(4);
}}
function recompute() {{
  const v = {{}};
  for (const [n] of INPUTS) v[n] = Number(document.getElementById("in_" + n).value);
  const rows = [];
  for (const [n, label, expr] of FORMULAS) {{
    const names = Object.keys(v);
    v[n] = Number(Function(...names, '"use strict"; return (' + expr + ');')(...names.map(k => v[k])));
    rows.push("<tr><td>" + label + "</td><td class=v>" + fmt(v[n]) + "</td><td><code>" + expr + "</code></td></tr>");
  }}
  document.getElementById("out").innerHTML = rows.join("");
}}
const box = document.getElementById("inputs");
for (const [n, label, d] of INPUTS) {{
  const l = document.createElement("label");
  l.textContent = label + " (" + n + ")";
  const i = document.createElement("input");
  i.type = "number"; i.id = "in_" + n; i.value = d; i.addEventListener("input", recompute);
  l.appendChild(i); box.appendChild(l);
}}
recompute();
</script></body></html>
"""


def render(values: dict | None = None) -> str:
    vals = values or {k: d for k, _, d in INPUTS}
    inputs = [[k, html.escape(label), vals[k]] for k, label, _ in INPUTS]
    formulas = [[n, html.escape(label), expr] for n, label, expr in FORMULAS]
    return _PAGE.format(inputs=json.dumps(inputs), formulas=json.dumps(formulas))


def main():
    from ..parallel.pipeline_entry import megagpt_model

    print(render(inputs_from_config(megagpt_model(), TPS=662754, GPUS=8, PEAK=2.25e15, HOURS=24)), end="")


if __name__ == "__main__":
    main()
