"""Curriculum over difficulty levels and a test-case-graded coding environment for GRPO.

The reference pairs a fixed-cadence curriculum with a mastery gate
(tunix-delphi-rl/environments/curriculum.py) with an environment whose dense reward is the
fraction of test cases a program passes, evaluated per level as pass@k on held-out instances
(tunix-delphi-rl/environments/curriculum_env.py, tunix-delphi-rl/training/train_curriculum.py).
Here:

* ``Curriculum``: levels ``1..L``; level 1 starts unlocked. Each level keeps an exponential moving
  average of batch success. Every ``steps_per_level`` steps the next level unlocks if the top
  unlocked level's average reached ``promote_threshold``, or after ``max_holds`` windows without
  it. Sampling covers all unlocked levels: the top (frontier) level gets ``frontier_weight``, the
  others share the rest, and none goes below ``floor_weight``. Levels above ``graduate_threshold``
  fall to the floor so the batches go where the policy still improves. The state is a few numbers
  (``state_dict`` / ``load_state_dict`` for checkpoints).
* ``TestCaseEnv``: programs in the safe subset of ``rl.envs.run_program`` (no imports, no function
  definitions); a problem binds its inputs as assignments before the program. Reward = fraction of
  test cases whose printed output matches. Levels: arithmetic on one input, two inputs, a loop, a
  conditional in a loop, nested loops.
* ``pass_at_k``: the unbiased estimator ``1 - C(n - c, k) / C(n, k)`` over ``n`` samples with ``c``
  correct; ``evaluate_passk`` averages it per level.
"""

from __future__ import annotations

import math
import random
from collections.abc import Callable
from dataclasses import dataclass, field

from .envs import ProgramError, Task, run_program


@dataclass(frozen=True)
class CurriculumConfig:
    num_levels: int
    steps_per_level: int = 40
    promote_threshold: float = 0.7
    graduate_threshold: float = 0.95
    max_holds: int = 3
    ema_decay: float = 0.9
    frontier_weight: float = 0.5
    floor_weight: float = 0.05


class Curriculum:
    def __init__(self, cfg: CurriculumConfig):
        if cfg.num_levels < 1:
            raise ValueError("num_levels must be >= 1")
        self.cfg = cfg
        self.unlocked = 1
        self.ema = [0.0] * cfg.num_levels
        self.seen = [False] * cfg.num_levels
        self.step = 0
        self.holds = 0

    def weights(self) -> list[float]:
        """Sampling weight of each level (0 for locked levels), summing to 1."""
        c, k = self.cfg, self.unlocked
        if k == 1:
            return [1.0] + [0.0] * (c.num_levels - 1)
        w = [0.0] * c.num_levels
        rest = (1.0 - c.frontier_weight) / (k - 1)
        for lv in range(k):
            w[lv] = c.frontier_weight if lv == k - 1 else rest
            if self.seen[lv] and self.ema[lv] >= c.graduate_threshold:
                w[lv] = c.floor_weight
            w[lv] = max(w[lv], c.floor_weight)
        tot = sum(w)
        return [x / tot for x in w]

    def sample_level(self, rng: random.Random) -> int:
        """A 1-indexed level for the next batch."""
        return rng.choices(range(1, self.cfg.num_levels + 1), weights=self.weights())[0]

    def record(self, level: int, success: float) -> None:
        i = level - 1
        d = self.cfg.ema_decay
        self.ema[i] = success if not self.seen[i] else d * self.ema[i] + (1 - d) * success
        self.seen[i] = True

    def on_step(self) -> bool:
        """Advance the schedule by one training step; True when a level unlocked."""
        self.step += 1
        c = self.cfg
        if self.step % c.steps_per_level or self.unlocked >= c.num_levels:
            return False
        top = self.unlocked - 1
        if (self.seen[top] and self.ema[top] >= c.promote_threshold) or self.holds >= c.max_holds:
            self.unlocked += 1
            self.holds = 0
            return True
        self.holds += 1
        return False

    def state_dict(self) -> dict:
        return {"unlocked": self.unlocked, "ema": list(self.ema), "seen": list(self.seen), "step": self.step,
                "holds": self.holds}

    def load_state_dict(self, st: dict) -> None:
        self.unlocked, self.step, self.holds = int(st["unlocked"]), int(st["step"]), int(st["holds"])
        self.ema, self.seen = [float(x) for x in st["ema"]], [bool(x) for x in st["seen"]]


# ------------------------------------------------------------------------------------ environment
@dataclass
class Problem:
    level: int
    prompt: str
    tests: list[tuple[str, str]] = field(default_factory=list)  # (input assignments, expected output)
    reference: str = ""  # a program that passes every test


def _make(level: int, rng: random.Random, n_tests: int) -> Problem:
    if level == 1:
        a = rng.randint(2, 9)
        prompt, ref = f"print x times {a} plus 1", f"print(x * {a} + 1)"
        cases = [{"x": rng.randint(-50, 50)} for _ in range(n_tests)]
        expect = [str(cs["x"] * a + 1) for cs in cases]
    elif level == 2:
        prompt, ref = "print the larger of x and y minus the smaller", "if x > y:\n    print(x - y)\nelse:\n    print(y - x)"
        cases = [{"x": rng.randint(-99, 99), "y": rng.randint(-99, 99)} for _ in range(n_tests)]
        expect = [str(abs(cs["x"] - cs["y"])) for cs in cases]
    elif level == 3:
        prompt, ref = "print the sum of 1..n", "s = 0\nfor i in range(1, n + 1):\n    s = s + i\nprint(s)"
        cases = [{"n": rng.randint(1, 60)} for _ in range(n_tests)]
        expect = [str(cs["n"] * (cs["n"] + 1) // 2) for cs in cases]
    elif level == 4:
        m = rng.randint(2, 5)
        prompt = f"print how many of 1..n are divisible by {m}"
        ref = f"c = 0\nfor i in range(1, n + 1):\n    if i % {m} == 0:\n        c = c + 1\nprint(c)"
        cases = [{"n": rng.randint(1, 80)} for _ in range(n_tests)]
        expect = [str(cs["n"] // m) for cs in cases]
    elif level == 5:
        prompt = "print the number of pairs (i, j) with 1 <= i < j <= n and i + j even"
        ref = ("c = 0\nfor i in range(1, n + 1):\n    for j in range(i + 1, n + 1):\n        if (i + j) % 2 == 0:\n"
               "            c = c + 1\nprint(c)")
        cases = [{"n": rng.randint(2, 25)} for _ in range(n_tests)]
        expect = [str(sum(1 for i in range(1, cs["n"] + 1) for j in range(i + 1, cs["n"] + 1) if (i + j) % 2 == 0))
                  for cs in cases]
    else:
        raise ValueError(f"no level {level}")
    tests = [("".join(f"{k} = {v}\n" for k, v in cs.items()), e) for cs, e in zip(cases, expect)]
    text = f"# Level {level}: {prompt}. Inputs are already assigned. Write the program, then END\n"
    return Problem(level, text, tests, ref)


class TestCaseEnv:
    __test__ = False  # not a pytest class
    num_levels = 5

    def __init__(self, seed: int = 0, n_tests: int = 5):
        self.rng = random.Random(seed)
        self.n_tests = n_tests

    def sample(self, level: int) -> Problem:
        return _make(level, self.rng, self.n_tests)

    def held_out(self, level: int, n: int, seed: int = 10_000) -> list[Problem]:
        rng = random.Random(seed * 31 + level)
        return [_make(level, rng, self.n_tests) for _ in range(n)]

    @staticmethod
    def extract_program(completion: str) -> str:
        return completion.split("END", 1)[0]

    @staticmethod
    def reward(completion: str, problem: Problem) -> float:
        prog = TestCaseEnv.extract_program(completion)
        ok = 0
        for pre, want in problem.tests:
            try:
                out = run_program(pre + prog).strip()
            except (ProgramError, SyntaxError, ValueError, TypeError, ZeroDivisionError, RecursionError):
                continue
            ok += out == want
        return ok / max(len(problem.tests), 1)


def pass_at_k(n: int, c: int, k: int) -> float:
    """Probability that at least one of ``k`` samples (drawn without replacement from ``n`` with
    ``c`` correct) is correct."""
    if k > n:
        raise ValueError("k must be <= n")
    if n - c < k:
        return 1.0
    return 1.0 - math.comb(n - c, k) / math.comb(n, k)


def evaluate_passk(policy: Callable[[Problem], list[str]], problems: list, k: int,
                   solved: Callable[[str, object], bool] | None = None) -> dict[int, float]:
    """Per level, the mean pass@k over ``problems``; ``policy(problem)`` returns n >= k completions
    and a completion counts as correct when it passes every test (``solved(completion, problem)``;
    by default the test-case environment's full reward)."""
    ok = solved or (lambda o, p: TestCaseEnv.reward(o, p) == 1.0)
    by: dict[int, list[float]] = {}
    for p in problems:
        outs = policy(p)
        c = sum(bool(ok(o, p)) for o in outs)
        by.setdefault(p.level, []).append(pass_at_k(len(outs), c, k))
    return {lv: sum(v) / len(v) for lv, v in sorted(by.items())}


class CurriculumTaskSource:
    """The environment interface of ``rl.learner.GRPOLearner`` over a curriculum: ``sample`` draws a
    level and a problem (the problem rides in the task's ``answer``), ``reward`` grades a completion
    and remembers it under the problem's level, ``on_step`` (called by the learner after each update)
    records each level's mean batch reward and advances the schedule."""

    def __init__(self, env: TestCaseEnv, curriculum: Curriculum, seed: int = 0):
        self.env, self.cur = env, curriculum
        self.rng = random.Random(seed)
        self._batch: dict[int, list[float]] = {}

    def sample(self) -> Task:
        p = self.env.sample(self.cur.sample_level(self.rng))
        return Task(p.prompt, p)

    def reward(self, completion: str, problem: Problem) -> float:
        r = self.env.reward(completion, problem)
        self._batch.setdefault(problem.level, []).append(r)
        return r

    def on_step(self) -> bool:
        for lv, rs in self._batch.items():
            self.cur.record(lv, sum(rs) / len(rs))
        self._batch.clear()
        return self.cur.on_step()
