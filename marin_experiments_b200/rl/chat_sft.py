"""Conversational SFT of a Qwen3-family policy: stage one of the agentic ladder
(tunix-delphi-rl/launch_chat_sft.py, tunix-delphi-rl/training/chat_sft.py).

A base model learns a turn-taking format from chat data: every conversation is rendered as ChatML
and tokenized with a loss mask on the assistant turns only (``data.chat.encode_chat``), rows are
packed into fixed-length sequences (conversations back to back, split at the sequence length;
padding carries no loss), and the model trains on the masked next-token cross-entropy with AdamW.
``run_chat_sft`` returns the loss curve plus generations for held-out prompts before and after
training, so the effect (a bounded assistant turn that ends with the end marker instead of a
rambling continuation) is visible.
"""

from __future__ import annotations

import math
import random
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..data.chat import IM_END, encode_chat, render_chatml


@dataclass
class ChatSFTConfig:
    steps: int = 1000
    batch_size: int = 8
    lr: float = 1e-5
    weight_decay: float = 0.0
    warmup: int = 0
    max_seq_len: int = 1024
    max_grad_norm: float = 1.0
    seed: int = 0
    eval_tokens: int = 200
    eval_temperature: float = 0.0
    log_every: int = 0
    extra: dict = field(default_factory=dict)


def pack_conversations(conversations: list[list[dict]], tok, seq_len: int, pad_id: int = 0):
    """``(tokens [N, seq_len], loss_mask [N, seq_len])``: conversations encoded with assistant-only
    masks, concatenated and cut into rows; the mask marks tokens whose *prediction* is trained (the
    target at position t is token t + 1)."""
    ids, mask = [], []
    for conv in conversations:
        a, m = encode_chat(conv, tok)
        ids += a
        mask += m
    n_rows = max(1, math.ceil(len(ids) / seq_len))
    total = n_rows * seq_len
    ids = ids + [pad_id] * (total - len(ids))
    mask = mask + [0] * (total - len(mask))
    t = torch.tensor(ids, dtype=torch.long).view(n_rows, seq_len)
    m = torch.tensor(mask, dtype=torch.float32).view(n_rows, seq_len)
    return t, m


def masked_lm_loss(model, tokens: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Mean next-token cross-entropy over the masked target positions."""
    logits = model.forward_logits(tokens[:, :-1])
    tgt = tokens[:, 1:]
    w = mask[:, 1:]
    ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), tgt.reshape(-1), reduction="none")
    return (ce * w.reshape(-1)).sum() / w.sum().clamp_min(1.0)


@torch.no_grad()
def generate(model, tok, prompt: str, max_tokens: int, temperature: float = 0.0, seed: int = 0,
             stop: str = IM_END) -> str:
    """One assistant turn for ``prompt`` (a user message) from the model's reference forward;
    stops at the end marker."""
    text = render_chatml([{"role": "user", "content": prompt}], add_generation_prompt=True)
    ids = tok.encode(text)
    gen = torch.Generator().manual_seed(seed)
    out: list[int] = []
    dev = next(model.parameters()).device
    for _ in range(max_tokens):
        logits = model.forward_logits(torch.tensor([ids + out], device=dev))[0, -1].float().cpu()
        if temperature <= 0:
            nxt = int(logits.argmax())
        else:
            nxt = int(torch.multinomial(torch.softmax(logits / temperature, -1), 1, generator=gen))
        out.append(nxt)
        if tok.decode(out).endswith(stop):
            break
    return tok.decode(out)


def run_chat_sft(model, tok, conversations: list[list[dict]], cfg: ChatSFTConfig,
                 eval_prompts: list[str] = ()) -> dict:
    """Train ``model`` on ``conversations``; returns ``{"losses", "before", "after"}``."""
    dev = next(model.parameters()).device
    before = [generate(model, tok, p, cfg.eval_tokens, cfg.eval_temperature, cfg.seed) for p in eval_prompts]
    tokens, mask = pack_conversations(conversations, tok, cfg.max_seq_len)
    tokens, mask = tokens.to(dev), mask.to(dev)
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=cfg.lr, weight_decay=cfg.weight_decay)
    rng = random.Random(cfg.seed)
    losses = []
    for step in range(cfg.steps):
        if cfg.warmup:
            for g in opt.param_groups:
                g["lr"] = cfg.lr * min(1.0, (step + 1) / cfg.warmup)
        rows = [rng.randrange(tokens.shape[0]) for _ in range(cfg.batch_size)]
        loss = masked_lm_loss(model, tokens[rows], mask[rows])
        opt.zero_grad(set_to_none=True)
        loss.backward()
        if cfg.max_grad_norm:
            torch.nn.utils.clip_grad_norm_(params, cfg.max_grad_norm)
        opt.step()
        losses.append(float(loss.detach()))
        if cfg.log_every and step % cfg.log_every == 0:
            print(f"[chat_sft] step={step} loss={losses[-1]:.4f}", flush=True)
    after = [generate(model, tok, p, cfg.eval_tokens, cfg.eval_temperature, cfg.seed) for p in eval_prompts]
    return {"losses": losses, "before": before, "after": after}


# ------------------------------------------------------------------ transcript (segment) SFT
def pack_segments(transcripts: list[list[tuple[str, int]]], tok, seq_len: int, pad_id: int = 0):
    """Rows of ``seq_len`` tokens from transcripts given as ``[(text, trained)]`` segments (the
    execution-format warm-up of tunix-delphi-rl/training/agentic_sft.py): each transcript is
    encoded segment by segment, so a trained segment's tokens are exactly its own; one transcript
    per row (cut at ``seq_len``), padding untrained. The mask marks the targets that are trained."""
    rows, masks = [], []
    for segs in transcripts:
        ids, m = [], []
        for text, trained in segs:
            enc = tok.encode(text)
            ids += enc
            m += [int(bool(trained))] * len(enc)
        ids, m = ids[:seq_len], m[:seq_len]
        rows.append(ids + [pad_id] * (seq_len - len(ids)))
        masks.append(m + [0] * (seq_len - len(m)))
    return torch.tensor(rows, dtype=torch.long), torch.tensor(masks, dtype=torch.float32)


def run_segment_sft(model, tok, transcripts: list[list[tuple[str, int]]], cfg: ChatSFTConfig) -> list[float]:
    """Masked next-token SFT over segment transcripts; returns the loss curve."""
    dev = next(model.parameters()).device
    tokens, mask = pack_segments(transcripts, tok, cfg.max_seq_len)
    tokens, mask = tokens.to(dev), mask.to(dev)
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=cfg.lr, weight_decay=cfg.weight_decay)
    rng = random.Random(cfg.seed)
    losses = []
    for step in range(cfg.steps):
        if cfg.warmup:
            for g in opt.param_groups:
                g["lr"] = cfg.lr * min(1.0, (step + 1) / cfg.warmup)
        rows = [rng.randrange(tokens.shape[0]) for _ in range(min(cfg.batch_size, tokens.shape[0]))]
        loss = masked_lm_loss(model, tokens[rows], mask[rows])
        opt.zero_grad(set_to_none=True)
        loss.backward()
        if cfg.max_grad_norm:
            torch.nn.utils.clip_grad_norm_(params, cfg.max_grad_norm)
        opt.step()
        losses.append(float(loss.detach()))
    return losses


@torch.no_grad()
def complete(model, tok, text: str, max_tokens: int, stops: tuple[str, ...] = ("\nEND",)) -> str:
    """Greedy continuation of raw ``text`` (base-model prompting), cut after the first stop string."""
    ids = tok.encode(text)
    out: list[int] = []
    dev = next(model.parameters()).device
    for _ in range(max_tokens):
        logits = model.forward_logits(torch.tensor([ids + out], device=dev))[0, -1]
        out.append(int(logits.argmax()))
        s = tok.decode(out)
        if any(st in s for st in stops):
            break
    return tok.decode(out)
