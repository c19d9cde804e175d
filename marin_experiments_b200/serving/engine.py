"""Batched text generation over a Qwen3 model with a KV cache (the role of the tunix Sampler behind
tunix-delphi-rl/serving/serve.py:334-420).

GPU path, per layer: RMSNorm -> one fused q|k|v GEMM -> per-head RMSNorm + RoPE at each row's
position -> KV-cache append -> attention (prefill: tcgen05 flash attention over the prompt;
decode: split-K attention of the new token over its cache) -> output GEMM with the residual in the
epilogue -> RMSNorm -> SwiGLU MLP GEMMs with the residual in the epilogue. Prompts are prefilled one
at a time; decode steps run every active sequence together, and a decode step for a given batch size
is captured once as a CUDA graph and replayed. Sampling: temperature, nucleus (top-p), per-request
seed; generation stops at end-of-document, ``max_tokens`` or a stop string.

CPU path: the model's fp32 reference forward over the whole sequence at every step (no cache) --
the oracle the GPU path is tested against.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..models.qwen3 import Qwen3Model


@dataclass
class SamplingParams:
    max_tokens: int = 64
    temperature: float = 0.8
    top_p: float = 1.0
    seed: int = 0
    stop: tuple[str, ...] = ()


def sample_next(logits: torch.Tensor, p: SamplingParams, gen: torch.Generator) -> torch.Tensor:
    """``logits [B, V]`` -> token ids ``[B]`` (greedy at temperature 0)."""
    if p.temperature <= 0:
        return logits.argmax(-1)
    probs = torch.softmax(logits.float() / p.temperature, dim=-1)
    if p.top_p < 1.0:
        sp, si = probs.sort(-1, descending=True)
        keep = sp.cumsum(-1) - sp < p.top_p
        sp = sp * keep
        probs = torch.zeros_like(probs).scatter(-1, si, sp)
    return torch.multinomial(probs / probs.sum(-1, keepdim=True), 1, generator=gen).squeeze(-1)


class Engine:
    def __init__(self, model: Qwen3Model, tokenizer, *, device=None, max_batch: int = 8, max_len: int | None = None,
                 use_graphs: bool = True):
        self.model = model
        self.tok = tokenizer
        self.cfg = model.cfg
        self.device = torch.device(device or next(model.parameters()).device)
        self.max_batch = max_batch
        self.max_len = max_len or min(self.cfg.max_seq_len, 4096)
        self.cuda = self.device.type == "cuda"
        self.use_graphs = use_graphs and self.cuda
        self.ready = False
        if self.cuda:
            self._prepare_cuda()
        self.ready = True

    # ------------------------------------------------------------------------------- setup
    def _prepare_cuda(self):
        c, dev = self.cfg, self.device
        bf = torch.bfloat16
        self.layers = []
        for L in self.model.layers:
            self.layers.append({
                "attn_norm": L.attn_norm.detach().float().to(dev), "mlp_norm": L.mlp_norm.detach().float().to(dev),
                "q_norm": L.q_norm.detach().float().contiguous().to(dev),
                "k_norm": L.k_norm.detach().float().contiguous().to(dev),
                "w_qkv": torch.cat([L.w_q, L.w_k, L.w_v], 0).detach().to(dev, bf).contiguous(),
                "w_o": L.w_o.detach().to(dev, bf).contiguous(),
                "w_gate_up": L.w_gate_up.detach().to(dev, bf).contiguous(),
                "w_down": L.w_down.detach().to(dev, bf).contiguous(),
            })
        self.embed = self.model.embed.detach().to(dev, bf).contiguous()
        self.head = self.model.head_weight().detach().to(dev, bf).contiguous()
        self.final_norm = self.model.final_norm.detach().float().to(dev)
        cos, sin = self.model.rope(dev)
        self.cos, self.sin = cos.contiguous(), sin.contiguous()
        shape = (self.max_batch, self.max_len, c.num_kv_heads, c.head_dim)
        self.kc = [torch.zeros(shape, dtype=bf, device=dev) for _ in range(c.num_layers)]
        self.vc = [torch.zeros(shape, dtype=bf, device=dev) for _ in range(c.num_layers)]
        self.nsplit = max(1, min(32, (148 * 2) // max(1, self.max_batch * c.num_kv_heads)))
        self.graphs: dict[int, tuple] = {}

    # ------------------------------------------------------------------------ GPU forward
    def _layer(self, x, W, li, pos, row_seq, prefill_len=None):
        from ..ops import api as ops
        from ..ops._ext import err_flag, ext

        c = self.cfg
        t = x.shape[0]
        nq, nk = c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim
        h = ops.rms_gated_norm(x, W["attn_norm"], c.norm_eps)
        qkv = ops.linear(h, W["w_qkv"])
        q = torch.empty(t, c.num_heads, c.head_dim, dtype=torch.bfloat16, device=x.device)
        k = torch.empty(t, c.num_kv_heads, c.head_dim, dtype=torch.bfloat16, device=x.device)
        ext().head_norm_rope(qkv[:, :nq], c.num_heads, c.head_dim, W["q_norm"], c.norm_eps, pos, self.cos, self.sin, q)
        ext().head_norm_rope(qkv[:, nq:nq + nk], c.num_kv_heads, c.head_dim, W["k_norm"], c.norm_eps, pos, self.cos,
                             self.sin, k)
        v = qkv[:, nq + nk:].view(t, c.num_kv_heads, c.head_dim)
        ext().kv_append(k, v, self.kc[li], self.vc[li], pos, row_seq)
        o = torch.empty(t, c.num_heads, c.head_dim, dtype=torch.bfloat16, device=x.device)
        scale = 1.0 / math.sqrt(c.head_dim)
        if prefill_len is not None:  # one sequence, causal over the prompt
            lse = torch.empty(t, c.num_heads, dtype=torch.float32, device=x.device)
            if c.head_dim in (64, 96, 128):
                ext().flash_fwd_sm100(q, k, v, o, lse, None, 1, t, 0, scale, err_flag(x.device), None)
            else:
                ext().flash_fwd(q, k, v, o, lse, None, 1, t, 0, scale)
        else:
            b = t
            ml = torch.empty(b, c.num_heads, self.nsplit, 2, dtype=torch.float32, device=x.device)
            acc = torch.empty(b, c.num_heads, self.nsplit, c.head_dim, dtype=torch.float32, device=x.device)
            kc = self.kc[li][:b] if row_seq is None else self.kc[li]
            vc = self.vc[li][:b] if row_seq is None else self.vc[li]
            ext().decode_attention(q, kc, vc, pos + 1, scale, self.nsplit, ml, acc, o)
        x = ops.linear(o.view(t, nq), W["w_o"], residual=x)
        h = ops.rms_gated_norm(x, W["mlp_norm"], c.norm_eps)
        return ops.dense_mlp(h, W["w_gate_up"], W["w_down"], glu=True, act="silu", residual=x)

    def _logits(self, x):
        from ..ops import api as ops

        h = ops.rms_gated_norm(x, self.final_norm, self.cfg.norm_eps)
        return ops.linear(h, self.head).float()

    @torch.no_grad()
    def _prefill(self, ids: list[int], slot: int) -> torch.Tensor:
        from ..ops import api as ops

        dev = self.device
        t = len(ids)
        tok = torch.tensor(ids, dtype=torch.long, device=dev)
        pos = torch.arange(t, dtype=torch.int32, device=dev)
        seq = torch.full((t,), slot, dtype=torch.int32, device=dev)
        x = ops.embed(tok, self.embed)
        for li, W in enumerate(self.layers):
            x = self._layer(x, W, li, pos, seq, prefill_len=t)
        return self._logits(x[-1:])

    def _decode_eager(self, tok, pos):
        from ..ops import api as ops

        x = ops.embed(tok, self.embed)
        for li, W in enumerate(self.layers):
            x = self._layer(x, W, li, pos, None)
        return self._logits(x)

    @torch.no_grad()
    def _decode(self, tok: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """One token for each of the first ``B`` cache slots (row b = slot b)."""
        b = tok.shape[0]
        if not self.use_graphs:
            return self._decode_eager(tok, pos)
        g = self.graphs.get(b)
        if g is None:
            st_tok, st_pos = tok.clone(), pos.clone()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                self._decode_eager(st_tok, st_pos)  # warm-up outside capture (tensor maps, allocator)
            torch.cuda.current_stream().wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = self._decode_eager(st_tok, st_pos)
            g = (graph, st_tok, st_pos, out)
            self.graphs[b] = g
        graph, st_tok, st_pos, out = g
        st_tok.copy_(tok)
        st_pos.copy_(pos)
        graph.replay()
        return out

    # ----------------------------------------------------------------------------- public
    @torch.no_grad()
    def generate(self, prompts: list[str], *, max_tokens: int | None = None, temperature: float = 0.8,
                 top_p: float = 1.0, seed: int = 0, stop: list[str] | None = None) -> list[str]:
        p = SamplingParams(max_tokens=max_tokens or 64, temperature=temperature, top_p=top_p, seed=seed,
                           stop=tuple(stop or ()))
        outs: list[str] = []
        for i in range(0, len(prompts), self.max_batch):
            outs += self._generate_batch(prompts[i:i + self.max_batch], p)
        return outs

    @torch.no_grad()
    def refresh_weights(self) -> None:
        """Copy the model's current weights into the engine's own (bf16) copies, in place: the
        buffers, the KV caches and any captured decode graphs stay valid, so an RL learner can
        sample from its latest policy every step without rebuilding the engine. The CPU path reads
        the model directly and has nothing to copy."""
        if not self.cuda:
            return
        for W, L in zip(self.layers, self.model.layers):
            W["attn_norm"].copy_(L.attn_norm.detach().float())
            W["mlp_norm"].copy_(L.mlp_norm.detach().float())
            W["q_norm"].copy_(L.q_norm.detach().float())
            W["k_norm"].copy_(L.k_norm.detach().float())
            W["w_qkv"].copy_(torch.cat([L.w_q, L.w_k, L.w_v], 0).detach())
            W["w_o"].copy_(L.w_o.detach())
            W["w_gate_up"].copy_(L.w_gate_up.detach())
            W["w_down"].copy_(L.w_down.detach())
        self.embed.copy_(self.model.embed.detach())
        self.head.copy_(self.model.head_weight().detach())
        self.final_norm.copy_(self.model.final_norm.detach().float())

    def generate_ids(self, prompts: list[list[int]], params: SamplingParams) -> list[list[int]]:
        """The sampled token ids of each prompt (end-of-document not included, stop strings not cut):
        what a learner trains on, with no re-tokenisation of decoded text."""
        outs: list[list[int]] = []
        for i in range(0, len(prompts), self.max_batch):
            outs += self._generate_ids_batch([list(x) or [self.tok.eos_id] for x in prompts[i:i + self.max_batch]],
                                             params)
        return outs

    def _generate_batch(self, prompts: list[str], p: SamplingParams) -> list[str]:
        new = self._generate_ids_batch([self.tok.encode(s) or [self.tok.eos_id] for s in prompts], p)
        texts = [self.tok.decode(x) for x in new]
        for j, s in enumerate(texts):
            for st in p.stop:
                k = s.find(st)
                if k >= 0:
                    s = s[:k]
            texts[j] = s
        return texts

    def _generate_ids_batch(self, ids: list[list[int]], p: SamplingParams) -> list[list[int]]:
        for x in ids:
            if len(x) + p.max_tokens > self.max_len:
                raise ValueError(f"prompt of {len(x)} tokens + {p.max_tokens} new exceeds max_len {self.max_len}")
        gen = torch.Generator(device=self.device).manual_seed(p.seed)
        b = len(ids)
        new: list[list[int]] = [[] for _ in range(b)]
        done = [False] * b
        if self.cuda:
            first = torch.cat([self._prefill(x, slot) for slot, x in enumerate(ids)], 0)
            tok = sample_next(first, p, gen)
            pos = torch.tensor([len(x) for x in ids], dtype=torch.int32, device=self.device)
        else:
            seqs = [list(x) for x in ids]
            tok = torch.stack([sample_next(self.model.forward_reference(torch.tensor([s]))[:, -1], p, gen)[0]
                               for s in seqs])
        for step in range(p.max_tokens):
            t_host = tok.tolist()
            for j in range(b):
                if done[j]:
                    continue
                if t_host[j] == self.tok.eos_id:
                    done[j] = True
                    continue
                new[j].append(t_host[j])
                if p.stop and any(s in self.tok.decode(new[j]) for s in p.stop):
                    done[j] = True
            if all(done) or step == p.max_tokens - 1:
                break
            if self.cuda:
                logits = self._decode(tok, pos)
                pos = pos + 1
            else:
                for j in range(b):
                    seqs[j].append(t_host[j])
                logits = torch.cat([self.model.forward_reference(torch.tensor([s]))[:, -1] for s in seqs], 0)
            tok = sample_next(logits, p, gen)
        return new
