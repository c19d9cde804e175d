"""RL environments with programmatic rewards (tunix-delphi-rl/environments/*.py).

* ``CalculatorEnv``: multiplication problems; reward 1 for the exact product as the last integer of
  the completion, with partial credit for the fraction of matching trailing digits.
* ``run_program``: a small interpreter for a safe Python subset (assignments, arithmetic,
  comparisons, ``if``/``while``/``for range``, ``print``), walked over the ``ast`` with a step limit --
  the role the reference's micropython interpreter plays (tunix-delphi-rl/environments/micropython.py).
  Programs can only compute and print; names outside the whitelist raise.
* ``CodingEnv``: tasks with a gold output; the completion's program (text up to ``END``) is run and
  rewarded 1 for an exact output match, else by output similarity.
"""

from __future__ import annotations

import ast
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


_ALLOWED_CALLS = {"print", "range", "abs", "min", "max", "len", "str", "int"}


def run_program(src: str, max_steps: int = 10_000) -> str:
    """Execute a program of the safe subset; returns its printed output."""
    tree = ast.parse(src, mode="exec")
    env: dict = {}
    out: list[str] = []
    steps = [0]

    def tick():
        steps[0] += 1
        if steps[0] > max_steps:
            raise ProgramError("step limit")

    def ev(n):
        tick()
        if isinstance(n, ast.Constant) and isinstance(n.value, (int, float, str, bool)):
            return n.value
        if isinstance(n, ast.Name):
            if n.id not in env:
                raise ProgramError(f"undefined {n.id}")
            return env[n.id]
        if isinstance(n, ast.BinOp):
            a, b = ev(n.left), ev(n.right)
            ops = {ast.Add: lambda: a + b, ast.Sub: lambda: a - b, ast.Mult: lambda: a * b,
                   ast.FloorDiv: lambda: a // b, ast.Mod: lambda: a % b, ast.Div: lambda: a / b,
                   ast.Pow: lambda: a ** b if abs(b) < 64 else (_ for _ in ()).throw(ProgramError("pow"))}
            if type(n.op) not in ops:
                raise ProgramError("operator")
            return ops[type(n.op)]()
        if isinstance(n, ast.UnaryOp) and isinstance(n.op, (ast.USub, ast.Not)):
            v = ev(n.operand)
            return -v if isinstance(n.op, ast.USub) else not v
        if isinstance(n, ast.Compare):
            left = ev(n.left)
            for op, rhs in zip(n.ops, n.comparators):
                right = ev(rhs)
                fn = {ast.Lt: left < right, ast.LtE: left <= right, ast.Gt: left > right, ast.GtE: left >= right,
                      ast.Eq: left == right, ast.NotEq: left != right}.get(type(op))
                if fn is None:
                    raise ProgramError("comparison")
                if not fn:
                    return False
                left = right
            return True
        if isinstance(n, ast.BoolOp):
            vals = [ev(v) for v in n.values]
            return all(vals) if isinstance(n.op, ast.And) else any(vals)
        if isinstance(n, ast.Call) and isinstance(n.func, ast.Name) and n.func.id in _ALLOWED_CALLS and not n.keywords:
            args = [ev(a) for a in n.args]
            if n.func.id == "print":
                out.append(" ".join(str(a) for a in args))
                return None
            if n.func.id == "range" and len(args) <= 3:
                r = range(*args)
                if len(r) > max_steps:
                    raise ProgramError("range too long")
                return r
            return {"abs": abs, "min": min, "max": max, "len": len, "str": str, "int": int}[n.func.id](*args)
        raise ProgramError(f"unsupported expression {type(n).__name__}")

    def ex(body):
        for st in body:
            tick()
            if isinstance(st, ast.Assign) and len(st.targets) == 1 and isinstance(st.targets[0], ast.Name):
                env[st.targets[0].id] = ev(st.value)
            elif isinstance(st, ast.AugAssign) and isinstance(st.target, ast.Name):
                env[st.target.id] = ev(ast.BinOp(ast.Name(st.target.id, ast.Load()), st.op, st.value))
            elif isinstance(st, ast.Expr):
                ev(st.value)
            elif isinstance(st, ast.If):
                ex(st.body if ev(st.test) else st.orelse)
            elif isinstance(st, ast.While):
                while ev(st.test):
                    ex(st.body)
            elif isinstance(st, ast.For) and isinstance(st.target, ast.Name) and not st.orelse:
                for v in ev(st.iter):
                    env[st.target.id] = v
                    ex(st.body)
            elif isinstance(st, ast.Pass):
                pass
            else:
                raise ProgramError(f"unsupported statement {type(st).__name__}")

    ex(tree.body)
    return "\n".join(out)


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
        except (ProgramError, SyntaxError, ValueError, TypeError, ZeroDivisionError, RecursionError):
            return 0.0
        if out == answer.strip():
            return 1.0
        return 0.5 * difflib.SequenceMatcher(None, out, answer).ratio()
