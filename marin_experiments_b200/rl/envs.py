"""RL environments with programmatic rewards (tunix-delphi-rl/environments/*.py).

* ``CalculatorEnv``: multiplication problems; reward 1 for the exact product as the last integer of
  the completion, with partial credit for the fraction of matching trailing digits.
* ``run_program``: a program's output from the sandboxed Python-subset interpreter ``rl.micropy``
  (the role of tunix-delphi-rl/environments/micropython.py); programs can only compute and print.
* ``CodingEnv``: tasks with a gold output; the completion's program (text up to ``END``) is run and
  rewarded 1 for an exact output match, else by output similarity.
"""

from __future__ import annotations

import difflib
import random
import re
from dataclasses import dataclass


@dataclass
class Task:
    prompt: str
    answer: str


class CalculatorEnv:
    def __init__(self, digits: tuple[int, int] = (2, 2), seed: int = 0):
        self.digits, self.rng = digits, random.Random(seed)

    def sample(self) -> Task:
        a = self.rng.randrange(10 ** (self.digits[0] - 1), 10 ** self.digits[0])
        b = self.rng.randrange(10 ** (self.digits[1] - 1), 10 ** self.digits[1])
        return Task(f"Compute {a} * {b} =", str(a * b))

    @staticmethod
    def reward(completion: str, answer: str) -> float:
        nums = re.findall(r"-?\d+", completion)
        if not nums:
            return 0.0
        got = nums[-1]
        if got == answer:
            return 1.0
        k = 0
        while k < min(len(got), len(answer)) and got[-1 - k] == answer[-1 - k]:
            k += 1
        return 0.5 * k / len(answer)


class ProgramError(Exception):
    pass


def run_program(src: str, max_steps: int = 10_000) -> str:
    """Run a program in the sandboxed interpreter (``rl.micropy``) and return its printed output
    without the final newline; a program that fails raises ``ProgramError`` with the interpreter's
    ``"Kind: message"``."""
    from .micropy import run

    r = run(src, max_steps=max_steps)
    if not r.ok:
        raise ProgramError(r.error)
    return r.stdout[:-1] if r.stdout.endswith("\n") else r.stdout


class CodingEnv:
    TASKS = [("print the sum of 17 and 25", "42"), ("print the numbers 1 to 3, one per line", "1\n2\n3"),
             ("print 7 factorial", "5040"), ("print whether 10 is even as True or False", "True")]

    def __init__(self, seed: int = 0):
        self.rng = random.Random(seed)

    def sample(self) -> Task:
        p, a = self.rng.choice(self.TASKS)
        return Task(f"# Task: {p}\n# Write a program, then END\n", a)

    @staticmethod
    def extract_program(completion: str) -> str:
        return completion.split("END", 1)[0]

    @staticmethod
    def reward(completion: str, answer: str) -> float:
        try:
            out = run_program(CodingEnv.extract_program(completion)).strip()
        except ProgramError:
            return 0.0
        if out == answer.strip():
            return 1.0
        return 0.5 * difflib.SequenceMatcher(None, out, answer).ratio()
