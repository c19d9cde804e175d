"""Tool-calling RL: chained multiplication through a calculator tool, multi-turn
(tunix-delphi-rl/environments/agentic_tools.py:1-817, tunix-delphi-rl/training/train_agentic.py).

A depth-d task multiplies d + 1 two-digit operands (11..99) with d dependent calculator calls: the
first call is ``CALC(a * b)``, every later one multiplies the previous tool result by the next
operand, and the episode ends with a final answer. Stage T0 is depth 1, T1 depth 2, T2 depth 3.
The surface is the plain ``CALC(x * y)`` line rather than JSON tool calls: a small base model writes
the line readily, and the skill being trained is copying operands (and tool results) correctly.

* ``chain_tasks(n, seed, depth)``: deterministic problem sets.
* ``parse_call`` (operands of the first ``CALC(x * y`` -- the closing parenthesis is optional, since
  a turn recorded without its stop token loses it) and ``call_closed`` (the strict form).
* ``CalcToolEnv``: the conversation state of one episode -- the few-shot system prompt and the task
  as the user turn; each assistant turn that contains a call is executed and answered with a
  ``Tool result: N`` turn, a turn without one is the final answer (or the turn budget runs out).
  Its terminal reward is copy-aware: +0.4 when the final answer repeats the last tool result
  (whatever the operands were) and +1.0 when it contains the gold product, both as standalone
  integers.
* ``arg_reward`` (+0.5: the first call carries the right operands) and ``format_reward`` (+0.1: the
  first call is closed) score the first assistant turn; ``metrics`` reports the tool-call rate, the
  operand accuracy and the solve ratio (total reward >= 1.0, which only the +1.0 term reaches).
* ``rollout(policy, env)``: one episode under a policy ``generate(text) -> str`` that continues the
  rendered conversation up to the end of its line.
"""

from __future__ import annotations

import random
import re
from collections.abc import Callable
from dataclasses import dataclass, field

SYSTEM_PROMPT = (
    "Use the calculator for every multiplication: write CALC(x * y) on its own line and read the\n"
    "Tool result. When all products are done, write the final number.\n"
    "Q: 12 * 13\n"
    "CALC(12 * 13)\n"
    "Tool result: 156\n"
    "156\n"
    "Q: 21 * 34 * 11\n"
    "CALC(21 * 34)\n"
    "Tool result: 714\n"
    "CALC(714 * 11)\n"
    "Tool result: 7854\n"
    "7854"
)

_CALL = re.compile(r"CALC\(\s*(-?\d+)\s*\*\s*(-?\d+)")
_CALL_CLOSED = re.compile(r"CALC\(\s*-?\d+\s*\*\s*-?\d+\s*\)")


@dataclass(frozen=True)
class ChainTask:
    prompt: str
    operands: tuple[int, ...]
    answer: str

    @property
    def depth(self) -> int:
        return len(self.operands) - 1


def chain_task(rng: random.Random, depth: int) -> ChainTask:
    ops = tuple(rng.randint(11, 99) for _ in range(depth + 1))
    prod = 1
    for v in ops:
        prod *= v
    return ChainTask("Q: " + " * ".join(map(str, ops)), ops, str(prod))


def chain_tasks(n: int, seed: int, depth: int) -> list[ChainTask]:
    rng = random.Random(seed)
    return [chain_task(rng, depth) for _ in range(n)]


def parse_call(text: str) -> tuple[int, int] | None:
    m = _CALL.search(text or "")
    return (int(m.group(1)), int(m.group(2))) if m else None


def call_closed(text: str) -> bool:
    return _CALL_CLOSED.search(text or "") is not None


def _has_int(text: str, value: str) -> bool:
    return re.search(rf"(?<!\d){re.escape(value)}(?!\d)", text or "") is not None


@dataclass
class CalcToolEnv:
    """One episode's state. ``turns`` holds (role, text) with roles user / assistant / tool."""

    task: ChainTask
    max_turns: int = 0  # assistant turns allowed; 0 -> depth + 1
    system: str = SYSTEM_PROMPT
    turns: list = field(default_factory=list)
    last_result: str | None = None
    done: bool = False
    calls: int = 0

    def __post_init__(self):
        if not self.max_turns:
            self.max_turns = self.task.depth + 1
        self.turns = [("user", self.task.prompt)]

    def render(self) -> str:
        """The text a policy continues: system prompt, the conversation, and a fresh line."""
        lines = [self.system]
        for role, text in self.turns:
            lines.append(f"Tool result: {text}" if role == "tool" else text)
        return "\n".join(lines) + "\n"

    def step(self, text: str) -> bool:
        """Record an assistant turn; execute its call if it has one. Returns whether the episode ended."""
        text = (text or "").split("\n")[0].strip()
        self.turns.append(("assistant", text))
        call = parse_call(text)
        n_assistant = sum(1 for r, _ in self.turns if r == "assistant")
        if call is not None and n_assistant < self.max_turns:
            self.calls += 1
            self.last_result = str(call[0] * call[1])
            self.turns.append(("tool", self.last_result))
            return False
        self.done = True
        return True

    @property
    def feedback(self) -> str | None:
        """The environment's text after the last assistant turn (``None`` once the episode ended)."""
        return None if self.done else f"Tool result: {self.turns[-1][1]}\n"

    @property
    def first_turn(self) -> str:
        return next((t for r, t in self.turns if r == "assistant"), "")

    @property
    def final_answer(self) -> str:
        return self.turns[-1][1] if self.done and self.turns[-1][0] == "assistant" else ""

    def reward(self) -> float:
        """Copy-aware terminal reward: +0.4 for repeating the last tool result, +1.0 for the gold."""
        ans = self.final_answer
        r = 0.0
        if self.last_result is not None and _has_int(ans, self.last_result):
            r += 0.4
        if _has_int(ans, self.task.answer):
            r += 1.0
        return r


def arg_reward(first_turn: str, task: ChainTask) -> float:
    ops = parse_call(first_turn)
    return 0.5 if ops is not None and set(ops) == set(task.operands[:2]) else 0.0


def format_reward(first_turn: str) -> float:
    return 0.1 if call_closed(first_turn) else 0.0


def total_reward(env: CalcToolEnv, with_format: bool = False) -> float:
    r = env.reward() + arg_reward(env.first_turn, env.task)
    return r + (format_reward(env.first_turn) if with_format else 0.0)


def metrics(envs: list[CalcToolEnv], rewards: list[float]) -> dict[str, float]:
    n = max(len(envs), 1)
    return {
        "tool/tool_call_rate": sum(call_closed(e.first_turn) for e in envs) / n,
        "tool/arg_acc": sum(arg_reward(e.first_turn, e.task) > 0 for e in envs) / n,
        "arithmetic/solve_ratio": sum(r >= 1.0 for r in rewards) / n,
    }


def rollout(policy: Callable[[str], str], task: ChainTask, max_turns: int = 0) -> CalcToolEnv:
    env = CalcToolEnv(task, max_turns=max_turns)
    while not env.done:
        env.step(policy(env.render()))
    return env
