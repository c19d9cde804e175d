"""Group-relative policy optimisation of a Qwen3 policy against an environment reward (the tunix
GRPO / Dr.GRPO learner role, tunix-delphi-rl/training/train_coding.py).

One ``step``: sample ``group_size`` completions per prompt (temperature sampling from the current
policy), score them with the environment, compute group advantages, and take one clipped
policy-gradient step (optionally several PPO-style epochs on the same rollouts) with global-norm
clipping.

Rollouts: by default each new token is sampled from the model's forward over the whole sequence so
far (simple, exact, quadratic in length). With ``use_engine`` they come from the serving engine
(``serving.engine.Engine``: KV cache, batched decode, CUDA graphs on a GPU), whose weight copies
are refreshed in place from the policy before every step, and completions end at end-of-document;
its token ids are trained as sampled.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .grpo import group_advantages, policy_loss, sequence_logprobs


@dataclass
class GRPOConfig:
    group_size: int = 4
    max_new_tokens: int = 16
    temperature: float = 1.0
    lr: float = 1e-4
    variant: str = "dr_grpo"
    clip_eps: float = 0.2
    epochs: int = 1
    max_grad_norm: float = 1.0
    seed: int = 0
    use_engine: bool = False


class GRPOLearner:
    def __init__(self, model, tokenizer, env, cfg: GRPOConfig | None = None):
        self.model, self.tok, self.env = model, tokenizer, env
        self.cfg = cfg or GRPOConfig()
        self.opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], lr=self.cfg.lr)
        self.gen = torch.Generator().manual_seed(self.cfg.seed)

    @torch.no_grad()
    def _sample(self, prompt_ids: list[int]) -> list[list[int]]:
        c = self.cfg
        if c.use_engine:
            from ..serving.engine import Engine, SamplingParams

            if getattr(self, "engine", None) is None:
                self.engine = Engine(self.model, self.tok, max_batch=c.group_size,
                                     max_len=min(self.model.cfg.max_seq_len, 4096))
                self._engine_calls = 0
            self.engine.refresh_weights()
            self._engine_calls += 1
            params = SamplingParams(max_tokens=c.max_new_tokens, temperature=c.temperature,
                                    seed=c.seed * 1_000_003 + self._engine_calls)
            return [x or [self.tok.eos_id] for x in self.engine.generate_ids([prompt_ids] * c.group_size, params)]
        seqs = [list(prompt_ids) for _ in range(c.group_size)]
        for _ in range(c.max_new_tokens):
            logits = self.model.forward_logits(torch.tensor(seqs))[:, -1].float()
            probs = torch.softmax(logits / max(c.temperature, 1e-5), -1)
            nxt = torch.multinomial(probs, 1, generator=self.gen).squeeze(1).tolist()
            for s, t in zip(seqs, nxt):
                s.append(t)
        return [s[len(prompt_ids):] for s in seqs]

    def step(self, n_prompts: int = 2) -> dict:
        c = self.cfg
        tasks = [self.env.sample() for _ in range(n_prompts)]
        rows, masks, rewards = [], [], []
        for t in tasks:
            p = self.tok.encode(t.prompt)
            for comp in self._sample(p):
                rows.append(p + comp)
                masks.append([0] * (len(p) - 1) + [1] * len(comp))
                rewards.append(self.env.reward(self.tok.decode(comp), t.answer))
        L = max(len(r) for r in rows)
        tokens = torch.tensor([r + [0] * (L - len(r)) for r in rows])
        mask = torch.tensor([m + [0] * (L - 1 - len(m)) for m in masks])
        rw = torch.tensor(rewards)
        adv = group_advantages(rw, c.group_size, c.variant)
        old = None
        for ep in range(c.epochs):
            logp = sequence_logprobs(self.model.forward_logits(tokens), tokens)
            if old is None:
                old = logp.detach()
            loss, met = policy_loss(logp, mask, adv, logp_old=old, clip_eps=c.clip_eps, variant=c.variant,
                                    max_len=c.max_new_tokens)
            self.opt.zero_grad(set_to_none=True)
            loss.backward()
            gn = torch.nn.utils.clip_grad_norm_(self.model.parameters(), c.max_grad_norm)
            self.opt.step()
        if hasattr(self.env, "on_step"):  # curriculum sources advance their schedule per update
            self.env.on_step()
        return {"loss": float(loss.detach()), "reward_mean": float(rw.mean()), "grad_norm": float(gn),
                "clip_frac": float(met["clip_frac"])}
