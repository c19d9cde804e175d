"""Multi-turn coding agent: write a program -> run it -> read the output -> revise
(tunix-delphi-rl/environments/coding_agent_env.py:1-954, tunix-delphi-rl/training/train_multiturn.py).

Each round the agent writes a program ended by a line holding only ``END``; the sandboxed
interpreter (``rl.micropy``) runs it and the environment answers with ``Tool result: <stdout>`` (or
``Tool result: Error: <kind>: <message>``). The episode ends as soon as a program's output equals the
gold output, or after ``max_rounds`` rounds. The interesting quantity is the gap between the
first-attempt solve rate and the best-of-rounds solve rate: repairing a program from its execution
feedback.

* ``coding_tasks(n, seed)``: tasks with a reference solution and the gold output it prints.
* ``extract_program``: the turn's text up to the ``END`` line (code fences dropped).
* ``grade`` / ``round_reward``: has-code (0.1), ran (0.3), output similarity (0.6 x ratio) and exact
  (1.0), so a group gets a graded signal before any round is exact; an exact round scores 2.0 and
  any non-exact one less than 1.0, so ``best >= SOLVED`` means solved.
* ``CodeAgentEnv``: the episode state; its reward is the best round's.
* ``make_bug``: a plausible wrong first attempt for a task (off-by-one range bound, swapped
  operator or comparison) whose output differs from the gold, and ``sft_transcript``: a transcript
  ``Task -> [buggy program -> Tool result ->] solution`` with per-segment loss masks, so repairing is
  in the fine-tuning data but rare -- the behaviour RL then amplifies.
* ``evaluate_multiturn`` (first / best solve rate and rounds used) and ``evaluate_passk`` /
  ``evaluate_repair_passk`` (k sampled first attempts, or k sampled fixes of a given buggy attempt).
"""

from __future__ import annotations

import difflib
import random
import re
from collections.abc import Callable
from dataclasses import dataclass, field

from . import micropy

SYSTEM_PROMPT = (
    "Write a short Python program for the task, then a line with only END. You will see its output\n"
    "as a line starting with \"Tool result:\". If it is wrong or failed, write a corrected program\n"
    "(again ending with END) until the output is right.\n"
    "Task: Print the product of the integers from 1 to 4.\n"
    "p = 1\n"
    "for i in range(1, 5):\n"
    "  p = p * i\n"
    "print(p)\n"
    "END\n"
    "Tool result: 24\n"
    "Task: Print the even numbers from 2 to 8 separated by spaces.\n"
    "print(' '.join([str(i) for i in range(2, 8, 2)]))\n"
    "END\n"
    "Tool result: 2 4 6\n"
    "print(' '.join([str(i) for i in range(2, 9, 2)]))\n"
    "END\n"
    "Tool result: 2 4 6 8"
)

W_HAS_CODE, W_RAN, W_PARTIAL, W_EXACT = 0.1, 0.3, 0.6, 1.0
SOLVED = 1.5  # an exact round scores 2.0; a non-exact one stays below 1.0
MAX_FEEDBACK = 400
RUN_STEPS = 200_000


@dataclass(frozen=True)
class CodingTask:
    prompt: str
    solution: str
    gold: str  # stdout of the solution (trailing newline included)


def _families(rng: random.Random) -> tuple[str, str]:
    k = rng.randrange(8)
    a, b = sorted(rng.sample(range(1, 30), 2))
    m = rng.randint(2, 7)
    if k == 0:
        return (f"Print the sum of the integers from {a} to {b} (inclusive).",
                f"s = 0\nfor i in range({a}, {b + 1}):\n  s = s + i\nprint(s)")
    if k == 1:
        return (f"Print the numbers from {a} to {b} (inclusive) separated by commas, with no spaces.",
                f"print(','.join([str(i) for i in range({a}, {b + 1})]))")
    if k == 2:
        n = rng.randint(3, 9)
        return (f"Print {n} factorial.", f"f = 1\nfor i in range(1, {n + 1}):\n  f = f * i\nprint(f)")
    if k == 3:
        return (f"Print how many integers from 1 to {b} are divisible by {m}.",
                f"c = 0\nfor i in range(1, {b + 1}):\n  if i % {m} == 0:\n    c = c + 1\nprint(c)")
    if k == 4:
        return (f"Print the squares of the integers from 1 to {m + 2}, one per line.",
                f"for i in range(1, {m + 3}):\n  print(i * i)")
    if k == 5:
        w = rng.choice(["banana", "compile", "tensor", "graft", "kernel"])
        return (f"Print the word '{w}' reversed.", f"print('{w}'[::-1])")
    if k == 6:
        return (f"Print the largest multiple of {m} that is at most {b + 20}.",
                f"x = {b + 20}\nwhile x % {m} != 0:\n  x = x - 1\nprint(x)")
    n = rng.randint(5, 12)
    return (f"Print the first {n} Fibonacci numbers (starting 1, 1) separated by spaces.",
            f"a = 1\nb = 1\nout = []\nfor i in range(0, {n}):\n  out.append(str(a))\n  t = a + b\n  a = b\n"
            f"  b = t\nprint(' '.join(out))")


def coding_task(rng: random.Random) -> CodingTask:
    prompt, sol = _families(rng)
    r = micropy.run(sol, max_steps=RUN_STEPS)
    if not r.ok:
        raise RuntimeError(f"reference solution failed: {r.error}\n{sol}")
    return CodingTask(prompt, sol, r.stdout)


def coding_tasks(n: int, seed: int, tiers: tuple[int, ...] | None = None) -> list[CodingTask]:
    """``n`` tasks; with ``tiers``, drawn from those tiers of ``rl.code_tasks`` instead."""
    if tiers is not None:
        from .code_tasks import sample_tasks

        return [CodingTask(t.prompt, t.solution, t.gold) for t in sample_tasks(n, seed, tuple(tiers))]
    rng = random.Random(seed)
    return [coding_task(rng) for _ in range(n)]


def extract_program(text: str) -> str:
    """The turn's program: its lines up to ``END`` (or up to a ``Tool result:`` / ``Task:`` line the
    policy wrote itself), code-fence lines dropped."""
    lines = []
    for ln in (text or "").split("\n"):
        if ln.strip() == "END" or ln.startswith(("Tool result:", "Task:")):
            break
        if ln.strip().startswith("```"):
            continue
        lines.append(ln)
    return "\n".join(lines).strip("\n")


def feedback(result: micropy.ExecResult, program: str) -> str:
    if not program.strip():
        return "(no program)"
    if not result.ok:
        return f"Error: {result.error}"[:MAX_FEEDBACK]
    if not result.stdout:
        return "(no output)"
    out = result.stdout
    if len(out) > MAX_FEEDBACK:
        out = out[:MAX_FEEDBACK] + "...(truncated)"
    return out.rstrip("\n")


def grade(result: micropy.ExecResult, program: str, gold: str) -> dict[str, float]:
    if not program.strip():
        return {"has_code": 0.0, "ran": 0.0, "partial": 0.0, "exact": 0.0}
    ran = float(result.ok)
    exact = float(result.ok and result.stdout == gold)
    partial = difflib.SequenceMatcher(None, result.stdout, gold).ratio() if result.ok else 0.0
    return {"has_code": 1.0, "ran": ran, "partial": partial, "exact": exact}


def round_reward(g: dict[str, float]) -> float:
    return W_HAS_CODE * g["has_code"] + W_RAN * g["ran"] + W_PARTIAL * g["partial"] + W_EXACT * g["exact"]


@dataclass
class CodeAgentEnv:
    task: CodingTask
    max_rounds: int = 4
    system: str = SYSTEM_PROMPT
    history: list = field(default_factory=list)  # (program, feedback) of finished rounds
    rewards: list = field(default_factory=list)
    solved_round: int = -1
    done: bool = False

    def render(self) -> str:
        parts = [f"{self.system}\nTask: {self.task.prompt}\n"]
        for prog, fb in self.history:
            parts.append(f"{prog}\nEND\nTool result: {fb}\n")
        return "".join(parts)

    def step(self, text: str) -> bool:
        prog = extract_program(text)
        res = micropy.run(prog, max_steps=RUN_STEPS) if prog.strip() else micropy.ExecResult("", False, "no program", 0)
        g = grade(res, prog, self.task.gold)
        self.rewards.append(round_reward(g))
        self.history.append((prog, feedback(res, prog)))
        if g["exact"]:
            self.solved_round = len(self.history) - 1
        self.done = bool(g["exact"]) or not prog.strip() or len(self.history) >= self.max_rounds
        return self.done

    @property
    def feedback(self) -> str | None:
        """The environment's text after the last program (``None`` once the episode ended)."""
        return None if self.done else f"Tool result: {self.history[-1][1]}\n"

    def reward(self) -> float:
        return max(self.rewards, default=0.0)

    @property
    def first_solved(self) -> bool:
        return self.solved_round == 0

    @property
    def solved(self) -> bool:
        return self.solved_round >= 0


_RANGE = re.compile(r"range\((\s*-?\d+\s*),(\s*-?\d+\s*)")


def make_bug(rng: random.Random, task: CodingTask) -> tuple[str, str] | None:
    """A wrong first attempt for ``task`` and its feedback: the first of a shuffled set of small
    mutations (upper range bound minus one, an operator or comparison swapped, a reversal
    slice turned into a truncation) whose output differs
    from the gold or which fails."""
    sol = task.solution
    cands = []
    m = _RANGE.search(sol)
    if m:
        cands.append(sol[:m.start()] + f"range({m.group(1)},{int(m.group(2)) - 1}" + sol[m.end():])
    for a, b in ((" + ", " - "), (" - ", " + "), (" * ", " + "), (" >= ", " > "), (" <= ", " < "),
                 (" == ", " != "), (" != ", " == "), ("[::-1]", "[:-1]")):
        if a in sol:
            cands.append(sol.replace(a, b, 1))
    rng.shuffle(cands)
    for c in cands:
        if c == sol:
            continue
        r = micropy.run(c, max_steps=RUN_STEPS)
        if not r.ok or r.stdout != task.gold:
            return c, feedback(r, c)
    return None


def sft_transcript(rng: random.Random, task: CodingTask, fix_prob: float = 0.3) -> list[tuple[str, int]]:
    """``[(text, trained)]``: the task line and tool results are context (0), programs are trained (1)."""
    segs = [(f"Task: {task.prompt}\n", 0)]
    if rng.random() < fix_prob:
        bug = make_bug(rng, task)
        if bug is not None:
            segs.append((f"{bug[0]}\nEND\n", 1))
            segs.append((f"Tool result: {bug[1]}\n", 0))
    segs.append((f"{task.solution}\nEND\n", 1))
    return segs


def run_episode(policy: Callable[[str], str], task: CodingTask, max_rounds: int = 4) -> CodeAgentEnv:
    env = CodeAgentEnv(task, max_rounds=max_rounds)
    while not env.done:
        env.step(policy(env.render()))
    return env


def evaluate_multiturn(policy: Callable[[str], str], tasks: list[CodingTask], max_rounds: int = 4) -> dict:
    envs = [run_episode(policy, t, max_rounds) for t in tasks]
    n = max(len(envs), 1)
    return {"first_solve": sum(e.first_solved for e in envs) / n, "best_solve": sum(e.solved for e in envs) / n,
            "mean_rounds": sum(len(e.history) for e in envs) / n, "envs": envs}


def _pass_at_k(n: int, c: int, k: int) -> float:
    if n - c < k:
        return 1.0
    p = 1.0
    for i in range(k):
        p *= (n - c - i) / (n - i)
    return 1.0 - p


def evaluate_passk(sample: Callable[[str, int], list[str]], tasks: list[CodingTask], k: int) -> dict:
    """``sample(prompt, k)`` returns k sampled first attempts; pass@1 and pass@k (unbiased estimator)."""
    p1 = pk = 0.0
    for t in tasks:
        env = CodeAgentEnv(t)
        outs = sample(env.render(), k)
        c = sum(micropy.run(extract_program(o), max_steps=RUN_STEPS).stdout == t.gold for o in outs)
        p1 += _pass_at_k(len(outs), c, 1)
        pk += _pass_at_k(len(outs), c, k)
    n = max(len(tasks), 1)
    return {"pass@1": p1 / n, f"pass@{k}": pk / n}


def evaluate_repair_passk(sample: Callable[[str, int], list[str]], tasks: list[CodingTask], k: int,
                          seed: int = 0) -> dict:
    """The same after a planted wrong first attempt and its feedback: can the policy fix it?"""
    rng = random.Random(seed)
    p1 = pk = 0.0
    m = 0
    for t in tasks:
        bug = make_bug(rng, t)
        if bug is None:
            continue
        env = CodeAgentEnv(t)
        env.history.append(bug)
        outs = sample(env.render(), k)
        c = sum(micropy.run(extract_program(o), max_steps=RUN_STEPS).stdout == t.gold for o in outs)
        p1 += _pass_at_k(len(outs), c, 1)
        pk += _pass_at_k(len(outs), c, k)
        m += 1
    m = max(m, 1)
    return {"repair_pass@1": p1 / m, f"repair_pass@{k}": pk / m, "tasks": m}
