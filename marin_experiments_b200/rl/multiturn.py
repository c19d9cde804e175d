"""Multi-turn GRPO: whole episodes (assistant turns interleaved with tool / interpreter output) as
one trained sequence per rollout (tunix-delphi-rl/training/train_multiturn.py:1-492,
tunix-delphi-rl/training/train_agentic.py:1-805).

An environment exposes ``render()`` (the opening text), ``step(text) -> done``, ``feedback`` (the
text it answers the last turn with, ``None`` once done) and ``reward()``; ``rl.tools.CalcToolEnv``
and ``rl.code_agent.CodeAgentEnv`` both do. A rollout keeps its own token transcript: the opening
prompt, then for each turn the sampled tokens (trained, mask 1) and the encoded feedback (context,
mask 0), and the policy is conditioned on that transcript rather than on a re-encoding of the
environment's text, so the trained tokens are exactly the sampled ones. A turn ends at the stop
string or after ``max_turn_tokens`` tokens. Each group of ``group_size`` episodes of one task gets
group-relative advantages from the episode rewards, and the clipped policy-gradient loss runs over
the assistant tokens of every turn. With ``use_engine`` each turn is decoded by the serving engine
(KV cache) from the transcript so far, its weights refreshed from the policy once per step.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch

from .grpo import group_advantages, policy_loss, sequence_logprobs
from .learner import GRPOConfig, GRPOLearner


@dataclass
class MultiTurnConfig(GRPOConfig):
    max_turn_tokens: int = 24
    stop: str = "\n"
    max_total_tokens: int = 512


class MultiTurnGRPO(GRPOLearner):
    def __init__(self, model, tokenizer, sample_task: Callable[[], object], make_env: Callable[[object], object],
                 cfg: MultiTurnConfig | None = None, reward_fn: Callable[[object], float] | None = None):
        self.sample_task, self.make_env = sample_task, make_env
        self.reward_fn = reward_fn or (lambda env: env.reward())
        super().__init__(model, tokenizer, None, cfg or MultiTurnConfig())

    def _engine(self):
        from ..serving.engine import Engine

        if getattr(self, "engine", None) is None:
            self.engine = Engine(self.model, self.tok, max_batch=1, max_len=min(self.model.cfg.max_seq_len, 4096))
            self._engine_calls = 0
        return self.engine

    @torch.no_grad()
    def _turn(self, ids: list[int]) -> list[int]:
        c = self.cfg
        if c.use_engine:  # KV-cache decode; the turn ends at the stop string, end of document or budget
            from ..serving.engine import SamplingParams

            budget = min(c.max_turn_tokens, c.max_total_tokens - len(ids), self.engine.max_len - len(ids))
            if budget <= 0:
                return []
            self._engine_calls += 1
            p = SamplingParams(max_tokens=budget, temperature=c.temperature, stop=(c.stop,),
                               seed=c.seed * 1_000_003 + self._engine_calls)
            return self.engine.generate_ids([ids], p)[0]
        out: list[int] = []
        for _ in range(c.max_turn_tokens):
            if len(ids) + len(out) >= c.max_total_tokens:
                break
            logits = self.model.forward_logits(torch.tensor([ids + out]))[0, -1].float()
            probs = torch.softmax(logits / max(c.temperature, 1e-5), -1)
            out.append(int(torch.multinomial(probs, 1, generator=self.gen)))
            if self.tok.decode(out).endswith(c.stop):
                break
        return out

    def rollout(self, task) -> tuple[list[int], list[int], object]:
        """One episode: (tokens, per-token train mask, finished environment)."""
        env = self.make_env(task)
        ids = self.tok.encode(env.render())
        mask = [0] * len(ids)
        while True:
            gen = self._turn(ids)
            ids, mask = ids + gen, mask + [1] * len(gen)
            text = self.tok.decode(gen)
            if env.step(text) or env.feedback is None or len(ids) >= self.cfg.max_total_tokens:
                break
            fb = ("" if text.endswith("\n") else "\n") + env.feedback
            enc = self.tok.encode(fb)
            ids, mask = ids + enc, mask + [0] * len(enc)
        return ids, mask, env

    def step(self, n_prompts: int = 2) -> dict:
        c = self.cfg
        if c.use_engine:  # this step's rollouts sample from the current weights
            self._engine().refresh_weights()
        rows, masks, rewards, envs = [], [], [], []
        for _ in range(n_prompts):
            task = self.sample_task()
            for _ in range(c.group_size):
                ids, m, env = self.rollout(task)
                rows.append(ids)
                masks.append(m)
                envs.append(env)
                rewards.append(float(self.reward_fn(env)))
        L = max(len(r) for r in rows)
        tokens = torch.tensor([r + [0] * (L - len(r)) for r in rows])
        mask = torch.tensor([m[1:] + [0] * (L - len(m)) for m in masks])
        rw = torch.tensor(rewards)
        adv = group_advantages(rw, c.group_size, c.variant)
        old = None
        for _ in range(c.epochs):
            logp = sequence_logprobs(self.model.forward_logits(tokens), tokens)
            if old is None:
                old = logp.detach()
            loss, met = policy_loss(logp, mask, adv, logp_old=old, clip_eps=c.clip_eps, variant=c.variant,
                                    max_len=L - 1)
            self.opt.zero_grad(set_to_none=True)
            loss.backward()
            gn = torch.nn.utils.clip_grad_norm_(self.model.parameters(), c.max_grad_norm)
            self.opt.step()
        turns = [sum(1 for i in range(1, len(m)) if m[i] and not m[i - 1]) for m in masks]
        return {"loss": float(loss.detach()), "reward_mean": float(rw.mean()), "grad_norm": float(gn),
                "clip_frac": float(met["clip_frac"]), "turns_mean": sum(turns) / len(turns),
                "trained_tokens": int(mask.sum()), "envs": envs}
