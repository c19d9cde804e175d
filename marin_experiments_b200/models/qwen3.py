"""Dense Qwen3 decoder for inference and serving (tunix-delphi-rl/models/delphi_qwen3.py:61-335,
tunix-delphi-rl/models/qwen3_loader.py:39-236, RoPE patch tunix-delphi-rl/models/delphi_patch.py:47-159).

Architecture: token embedding -> N x [RMSNorm -> attention (q/k/v projections, per-head RMSNorm of
q and k with learned scales, RoPE with theta and optional Llama-3 frequency scaling, causal GQA,
output projection) + residual -> RMSNorm -> SwiGLU MLP + residual] -> RMSNorm -> LM head (optionally
tied to the embedding).

Weights are held in the framework's layouts: gate/up rows block-interleaved (``ops.layout``) so the
SwiGLU runs in the GEMM epilogue. ``load_hf`` reads a Hugging Face ``Qwen3ForCausalLM`` snapshot
(``config.json`` + ``*.safetensors``) with a coverage check; ``models/qwen3_export.py`` writes it
back. On CUDA the forward uses the sm_100a kernels: tcgen05 GEMMs, tcgen05 flash attention for
prefill, split-K decode attention over the KV cache; on CPU the fp32 oracle ops.
"""

from __future__ import annotations

import glob
import json
import os
from dataclasses import dataclass

import torch
from torch import nn

from ..ops import reference as R
from ..ops.layout import gate_up_to_blocked_rows


@dataclass(frozen=True)
class Qwen3Config:
    vocab_size: int = 128256
    hidden_dim: int = 1024
    intermediate_dim: int = 4096
    num_layers: int = 11
    num_heads: int = 8
    num_kv_heads: int = 8
    head_dim: int = 128
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None  # {"factor", "low_freq_factor", "high_freq_factor", "original_max_position_embeddings"}
    norm_eps: float = 1e-5
    tie_embeddings: bool = False
    max_seq_len: int = 4096

    @staticmethod
    def from_hf(d: dict) -> "Qwen3Config":
        arch = d.get("architectures")
        if arch and list(arch) != ["Qwen3ForCausalLM"]:
            raise ValueError(f"expected Qwen3ForCausalLM, got {arch!r}")
        rs = d.get("rope_scaling")
        if rs is not None and rs.get("rope_type", rs.get("type")) not in (None, "llama3"):
            raise ValueError(f"unsupported rope_scaling {rs!r}")
        return Qwen3Config(vocab_size=d["vocab_size"], hidden_dim=d["hidden_size"],
                           intermediate_dim=d["intermediate_size"], num_layers=d["num_hidden_layers"],
                           num_heads=d["num_attention_heads"], num_kv_heads=d.get("num_key_value_heads",
                                                                                  d["num_attention_heads"]),
                           head_dim=d.get("head_dim", d["hidden_size"] // d["num_attention_heads"]),
                           rope_theta=float(d.get("rope_theta", 10000.0)), rope_scaling=rs,
                           norm_eps=float(d.get("rms_norm_eps", 1e-6)),
                           tie_embeddings=bool(d.get("tie_word_embeddings", False)),
                           max_seq_len=int(d.get("max_position_embeddings", 4096)))

    def to_hf(self) -> dict:
        d = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": self.vocab_size,
             "hidden_size": self.hidden_dim, "intermediate_size": self.intermediate_dim,
             "num_hidden_layers": self.num_layers, "num_attention_heads": self.num_heads,
             "num_key_value_heads": self.num_kv_heads, "head_dim": self.head_dim, "rope_theta": self.rope_theta,
             "rms_norm_eps": self.norm_eps, "tie_word_embeddings": self.tie_embeddings,
             "max_position_embeddings": self.max_seq_len, "hidden_act": "silu", "torch_dtype": "bfloat16"}
        if self.rope_scaling is not None:
            d["rope_scaling"] = dict(self.rope_scaling)
        return d

    def llama3(self) -> dict | None:
        rs = self.rope_scaling
        if rs is None:
            return None
        return {"scaling_factor": float(rs.get("factor", 8.0)), "low_freq_factor": float(rs.get("low_freq_factor", 1.0)),
                "high_freq_factor": float(rs.get("high_freq_factor", 4.0)),
                "original_max_position": int(rs.get("original_max_position_embeddings", 8192))}


class Qwen3Layer(nn.Module):
    def __init__(self, c: Qwen3Config):
        super().__init__()
        d, hd = c.hidden_dim, c.head_dim
        self.attn_norm = nn.Parameter(torch.ones(d))
        self.w_q = nn.Parameter(torch.empty(c.num_heads * hd, d))
        self.w_k = nn.Parameter(torch.empty(c.num_kv_heads * hd, d))
        self.w_v = nn.Parameter(torch.empty(c.num_kv_heads * hd, d))
        self.q_norm = nn.Parameter(torch.ones(hd))
        self.k_norm = nn.Parameter(torch.ones(hd))
        self.w_o = nn.Parameter(torch.empty(d, c.num_heads * hd))
        self.mlp_norm = nn.Parameter(torch.ones(d))
        self.w_gate_up = nn.Parameter(torch.empty(2 * c.intermediate_dim, d))  # block-interleaved
        self.w_down = nn.Parameter(torch.empty(d, c.intermediate_dim))


class Qwen3Model(nn.Module):
    def __init__(self, c: Qwen3Config):
        super().__init__()
        if c.intermediate_dim % 128:
            raise ValueError("intermediate_dim must be a multiple of 128 (block-interleaved gate/up)")
        self.cfg = c
        self.embed = nn.Parameter(torch.empty(c.vocab_size, c.hidden_dim))
        self.layers = nn.ModuleList([Qwen3Layer(c) for _ in range(c.num_layers)])
        self.final_norm = nn.Parameter(torch.ones(c.hidden_dim))
        self.lm_head = None if c.tie_embeddings else nn.Parameter(torch.empty(c.vocab_size, c.hidden_dim))
        self._rope = None

    def init_weights(self, seed: int = 0, std: float = 0.02) -> "Qwen3Model":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if p.dim() >= 2:
                    p.copy_(torch.randn(p.shape, generator=g) * std)
        return self

    def head_weight(self) -> torch.Tensor:
        return self.embed if self.lm_head is None else self.lm_head

    def rope(self, device):
        c = self.cfg
        if self._rope is None or self._rope[0].device != torch.device(device):
            self._rope = R.rope_cos_sin(c.max_seq_len, c.head_dim, c.rope_theta, device=device, llama3=c.llama3())
        return self._rope

    # ----------------------------------------------------------------------------- reference
    @torch.no_grad()
    def forward_reference(self, tokens: torch.Tensor) -> torch.Tensor:
        """fp32 logits ``[B, S, V]`` with plain torch ops (the oracle of the serving path)."""
        return self.forward_logits(tokens)

    def forward_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """Differentiable fp32 forward (policy-gradient training of small models)."""
        c = self.cfg
        b, s = tokens.shape
        x = self.embed.float()[tokens]
        cos, sin = self.rope(tokens.device)
        cos, sin = cos[:s], sin[:s]
        for L in self.layers:
            h = R.rms_norm(x, L.attn_norm, c.norm_eps)
            q = (h @ L.w_q.float().t()).view(b, s, c.num_heads, c.head_dim)
            k = (h @ L.w_k.float().t()).view(b, s, c.num_kv_heads, c.head_dim)
            v = (h @ L.w_v.float().t()).view(b, s, c.num_kv_heads, c.head_dim)
            q = R.apply_rope(R.rms_norm(q, L.q_norm, c.norm_eps), cos, sin)
            k = R.apply_rope(R.rms_norm(k, L.k_norm, c.norm_eps), cos, sin)
            o = R.attention(q, k, v).reshape(b, s, -1)
            x = x + o @ L.w_o.float().t()
            h = R.rms_norm(x, L.mlp_norm, c.norm_eps)
            z = h @ L.w_gate_up.float().t()
            from ..ops.layout import split_gate_up

            gg, uu = split_gate_up(z, c.intermediate_dim)
            x = x + (R.activation(gg, "silu") * uu) @ L.w_down.float().t()
        x = R.rms_norm(x, self.final_norm, c.norm_eps)
        return x @ self.head_weight().float().t()


# ---------------------------------------------------------------------------------- HF I/O
_HF_LAYER = {
    "input_layernorm.weight": "attn_norm",
    "self_attn.q_proj.weight": "w_q",
    "self_attn.k_proj.weight": "w_k",
    "self_attn.v_proj.weight": "w_v",
    "self_attn.q_norm.weight": "q_norm",
    "self_attn.k_norm.weight": "k_norm",
    "self_attn.o_proj.weight": "w_o",
    "post_attention_layernorm.weight": "mlp_norm",
    "mlp.down_proj.weight": "w_down",
}


def load_hf(model_dir: str, device="cpu", dtype=torch.bfloat16) -> Qwen3Model:
    """Build a ``Qwen3Model`` from a local Hugging Face snapshot; every checkpoint tensor must be
    consumed and every model parameter filled (the loader's coverage assertion)."""
    from safetensors.torch import load_file

    with open(os.path.join(model_dir, "config.json")) as f:
        cfg = Qwen3Config.from_hf(json.load(f))
    sd = {}
    for fn in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
        sd.update(load_file(fn))
    if not sd:
        raise FileNotFoundError(f"no safetensors under {model_dir}")
    with torch.device("meta"):
        model = Qwen3Model(cfg)
    model = model.to_empty(device=device)
    filled = set()
    used = set()

    def put(param: nn.Parameter, t: torch.Tensor, key: str, name: str):
        if tuple(t.shape) != tuple(param.shape):
            raise ValueError(f"{key}: shape {tuple(t.shape)} != {tuple(param.shape)}")
        with torch.no_grad():
            param.copy_(t.to(device=device, dtype=param.dtype))
        filled.add(name)
        used.add(key)

    put(model.embed, sd["model.embed_tokens.weight"], "model.embed_tokens.weight", "embed")
    put(model.final_norm, sd["model.norm.weight"], "model.norm.weight", "final_norm")
    if model.lm_head is not None:
        put(model.lm_head, sd["lm_head.weight"], "lm_head.weight", "lm_head")
    elif "lm_head.weight" in sd:
        used.add("lm_head.weight")
    for i, L in enumerate(model.layers):
        pre = f"model.layers.{i}."
        for hk, ours in _HF_LAYER.items():
            put(getattr(L, ours), sd[pre + hk], pre + hk, f"layers.{i}.{ours}")
        gate, up = sd[pre + "mlp.gate_proj.weight"], sd[pre + "mlp.up_proj.weight"]
        put(L.w_gate_up, gate_up_to_blocked_rows(gate.float(), up.float()), pre + "mlp.gate_proj.weight",
            f"layers.{i}.w_gate_up")
        used.add(pre + "mlp.up_proj.weight")
    missing = [n for n, _ in model.named_parameters() if n not in filled]
    unused = [k for k in sd if k not in used]
    if missing or unused:
        raise ValueError(f"checkpoint coverage mismatch: missing {missing[:8]}, unused {unused[:8]}")
    norms = ("attn_norm", "q_norm", "k_norm", "mlp_norm", "final_norm")
    for n, p in model.named_parameters():
        if any(n.endswith(k) for k in norms):
            p.data = p.data.float()
        else:
            p.data = p.data.to(dtype)
    return model


def param_count(c: Qwen3Config) -> int:
    d, i, hd = c.hidden_dim, c.intermediate_dim, c.head_dim
    per = d * hd * (c.num_heads * 2 + c.num_kv_heads * 2) + 3 * d * i + 2 * d + 2 * hd
    emb = c.vocab_size * d * (1 if c.tie_embeddings else 2)
    return c.num_layers * per + emb + d


