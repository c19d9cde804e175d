"""Staged single-turn arithmetic for GRPO on a base (non-chat) model
(tunix-delphi-rl/problems/arithmetic.py:1-389, tunix-delphi-rl/training/train_delphi.py:1-222).

A base model follows a format only when the demonstrations in front of the query are of the same
kind of task, so every stage carries its own few-shot block and the prompt ends exactly where the
number should come (``A:``, or ``x =`` for equations). The answer is the first (optionally signed)
integer of the completion.

Stages:

* 0 -- ``a + b`` with single digits;
* 1 -- ``a op b`` with ``op`` in ``+ - *`` and operands below 100 (subtraction ordered so the
  answer is not negative);
* 2 -- two operations with the usual precedence: ``a * b + c``, ``a + b * c``, ``(a + b) * c``,
  ``a - b + c``;
* 3 -- ``Solve for x: a*x + b = c`` with an integer (possibly negative) solution.

Rewards: ``answer_reward`` (1.0 for the gold), ``format_reward`` (0.1 when the completion starts
with an integer: the format is kept even when the value is wrong), ``proximity_reward`` (dense
partial credit ``0.5 / (1 + |error| / scale)`` with the scale set by the gold's magnitude, 0 for
an exact answer so it adds to ``answer_reward`` without double counting). ``group_metrics`` reports
the solve ratio and the share of groups solved by all and by none of their samples (groups that
give GRPO no signal).
"""

from __future__ import annotations

import random
import re

from .envs import Task

FEWSHOT = {
    0: "Q: 3 + 4 =\nA: 7\nQ: 8 + 1 =\nA: 9\nQ: 5 + 5 =\nA: 10\n",
    1: "Q: 23 + 48 =\nA: 71\nQ: 90 - 37 =\nA: 53\nQ: 12 * 7 =\nA: 84\n",
    2: "Q: 3 * 4 + 5 =\nA: 17\nQ: 2 + 6 * 3 =\nA: 20\nQ: (4 + 1) * 6 =\nA: 30\n",
    3: "Solve for x: 2*x + 3 = 11; x = 4\nSolve for x: 5*x - 2 = -12; x = -2\nSolve for x: 3*x + 0 = 21; x = 7\n",
}
STAGES = tuple(sorted(FEWSHOT))
_INT = re.compile(r"^\s*(-?\d+)")
_ANY_INT = re.compile(r"-?\d+")


def make_problem(stage: int, rng: random.Random) -> tuple[str, str]:
    """(query text, gold answer); the query is appended to the stage's few-shot block."""
    if stage == 0:
        a, b = rng.randint(0, 9), rng.randint(0, 9)
        return f"Q: {a} + {b} =\nA:", str(a + b)
    if stage == 1:
        a, b = rng.randint(0, 99), rng.randint(0, 99)
        op = rng.choice("+-*")
        if op == "-" and b > a:
            a, b = b, a
        return f"Q: {a} {op} {b} =\nA:", str(a + b if op == "+" else a - b if op == "-" else a * b)
    if stage == 2:
        a, b, c = rng.randint(1, 12), rng.randint(1, 12), rng.randint(1, 12)
        form = rng.randrange(4)
        expr, val = [(f"{a} * {b} + {c}", a * b + c), (f"{a} + {b} * {c}", a + b * c),
                     (f"({a} + {b}) * {c}", (a + b) * c), (f"{a} - {b} + {c}", a - b + c)][form]
        return f"Q: {expr} =\nA:", str(val)
    if stage == 3:
        a = rng.choice([v for v in range(-6, 10) if v not in (0, 1)])
        x = rng.randint(-9, 12)
        b = rng.randint(-20, 20)
        c = a * x + b
        lhs = f"{a}*x {'+' if b >= 0 else '-'} {abs(b)}"
        return f"Solve for x: {lhs} = {c}; x =", str(x)
    raise ValueError(f"no stage {stage}")


def build_prompt(stage: int, query: str) -> str:
    return FEWSHOT[stage] + query


def parse_answer(completion: str) -> int | None:
    m = _INT.match(completion or "")
    if m:
        return int(m.group(1))
    m = _ANY_INT.search((completion or "").split("\n")[0])
    return int(m.group(0)) if m else None


def answer_reward(completion: str, gold: str) -> float:
    v = parse_answer(completion)
    return 1.0 if v is not None and v == int(gold) else 0.0


def format_reward(completion: str) -> float:
    return 0.1 if _INT.match(completion or "") else 0.0


def proximity_reward(completion: str, gold: str) -> float:
    v = parse_answer(completion)
    g = int(gold)
    if v is None or v == g:
        return 0.0
    scale = max(1.0, abs(g) / 10.0)
    return 0.5 / (1.0 + abs(v - g) / scale)


def total_reward(completion: str, gold: str, dense: bool = True) -> float:
    r = answer_reward(completion, gold) + format_reward(completion)
    return r + (proximity_reward(completion, gold) if dense else 0.0)


def group_metrics(completions: list[str], golds: list[str], group_size: int) -> dict[str, float]:
    ok = [answer_reward(c, g) == 1.0 for c, g in zip(completions, golds)]
    groups = [ok[i:i + group_size] for i in range(0, len(ok), group_size)]
    n = max(len(groups), 1)
    return {"arith/solve_ratio": sum(ok) / max(len(ok), 1), "arith/solve_all": sum(all(g) for g in groups) / n,
            "arith/solve_none": sum(not any(g) for g in groups) / n}


class ArithmeticEnv:
    """``sample`` / ``reward`` for ``rl.learner.GRPOLearner``; ``stage`` can be changed between steps."""

    def __init__(self, stage: int = 0, seed: int = 0, dense: bool = True):
        self.stage, self.dense = stage, dense
        self.rng = random.Random(seed)

    def sample(self) -> Task:
        q, gold = make_problem(self.stage, self.rng)
        return Task(build_prompt(self.stage, q), gold)

    def reward(self, completion: str, answer: str) -> float:
        return total_reward(completion, answer, self.dense)
