"""A toy GRPO run that shows the learner learning in seconds on a CPU
(tunix-delphi-rl/examples/toy_cats.py:64-470).

A word-level tokenizer over a dozen words, a one-layer Qwen3 policy from random weights, prompts
that are a fixed opener, and a reward equal to the share of generated words that are ``cat``. A
few dozen Dr.GRPO steps drive the mean reward from chance (about one word in twelve) towards 1:
the whole loop -- sampling, group advantages, clipped policy gradient, optimizer -- has to work
for that to happen. ``train_toy`` returns the reward history.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .envs import Task
from .learner import GRPOConfig, GRPOLearner

WORDS = ("<pad>", "the", "a", "cat", "dog", "sat", "ran", "on", "mat", "big", "small", "and")


class WordTokenizer:
    """Space-separated words of ``WORDS``; unknown words map to ``<pad>``."""

    def __init__(self, words: tuple[str, ...] = WORDS):
        self.words = words
        self.index = {w: i for i, w in enumerate(words)}
        self.vocab_size = len(words)
        self.eos_id = 0

    def encode(self, text: str) -> list[int]:
        return [self.index.get(w, 0) for w in text.split()]

    def decode(self, ids: list[int]) -> str:
        return " ".join(self.words[i] for i in ids)


class CatEnv:
    """Prompts are ``the big``; the reward is the share of generated words equal to ``cat``."""

    def sample(self) -> Task:
        return Task("the big", "")

    @staticmethod
    def reward(completion: str, answer: str) -> float:
        w = completion.split()
        return sum(x == "cat" for x in w) / max(len(w), 1)


@dataclass
class ToyResult:
    rewards: list[float]
    first: float
    last: float


def toy_model(seed: int = 0):
    from ..models.qwen3 import Qwen3Config, Qwen3Model

    cfg = Qwen3Config(vocab_size=len(WORDS), hidden_dim=32, intermediate_dim=128, num_layers=1, num_heads=2,
                      num_kv_heads=1, head_dim=16, max_seq_len=64)
    return Qwen3Model(cfg).init_weights(seed)


def train_toy(steps: int = 40, seed: int = 0, lr: float = 1e-2, group_size: int = 8, max_new_tokens: int = 6,
              n_prompts: int = 2) -> ToyResult:
    torch.manual_seed(seed)
    learner = GRPOLearner(toy_model(seed), WordTokenizer(), CatEnv(),
                          GRPOConfig(group_size=group_size, max_new_tokens=max_new_tokens, lr=lr, seed=seed,
                                     max_grad_norm=1.0))
    hist = [learner.step(n_prompts=n_prompts)["reward_mean"] for _ in range(steps)]
    k = max(1, steps // 5)
    return ToyResult(hist, sum(hist[:k]) / k, sum(hist[-k:]) / k)


if __name__ == "__main__":
    r = train_toy()
    print(f"mean reward: first {r.first:.3f} -> last {r.last:.3f}")
