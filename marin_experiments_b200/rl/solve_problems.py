"""Function-writing problems graded on many test cases: nine levels of parameterised ``def solve``
families with public and hidden tests, for curriculum RL (tunix-delphi-rl/problems/coding_problems.py:93-1260,
tunix-delphi-rl/environments/curriculum_env.py:1-397).

A problem asks for ``def solve(...)``; the prompt shows its signature, a description and the
public tests, and the grade runs the submitted program on every public and hidden test through
the sandboxed interpreter (``rl.micropy``). A group of samples that each pass a different share of
the tests gets a spread of rewards even when no sample is perfect, which is the signal Dr.GRPO
needs early on. The expected output of a test is what the family's reference prints when run by
the same interpreter, so number and list formatting always match the engine the policy's program
runs in; a call is written out as a literal (``print(solve(3, [1, 2]))``), since the interpreter has
no starred arguments.

Levels (three families each, the later ones compositional: an intermediate result that is then
reduced or transformed, so a shaky first attempt tends to be partly right):

1. one integer in, arithmetic out;  2. two inputs, a branch;  3. a loop over ``range``;
4. lists (sum, count, extremes with an empty-list case);  5. strings;  6. loops with branches;
7. primes / sets / words then a reduction;  8. factorial, Collatz, an expression string;
9. gcd / lcm chains, a mode with ties, running balances.

Generators mix edge cases (empty lists, 0 and 1, negatives, duplicates, ties) with ordinary inputs
so a memorised constant fails the hidden tests. ``grade`` returns ``has_code`` (the program defines
``solve``), ``ran_ok`` (every test ran without an error), ``frac_passed`` and ``exact``;
``reward = 0.1 has_code + 0.2 ran_ok + 0.7 frac_passed``. ``feedback`` describes the first
failing public test for multi-turn repair. ``SolveProblemEnv`` has the ``sample(level)`` /
``held_out`` / ``reward`` interface of ``rl.curriculum.CurriculumTaskSource``.
"""

from __future__ import annotations

import random
import re
from collections.abc import Callable
from dataclasses import dataclass, field

from . import micropy

NUM_LEVELS = 9
GRADE_STEPS = 20_000
N_PUBLIC = 2
N_HIDDEN = 6
W_HAS_CODE, W_RAN_OK, W_FRAC = 0.1, 0.2, 0.7
_SOLVE = re.compile(r"^def solve\(", re.M)


@dataclass(frozen=True)
class Problem:
    id: str
    level: int
    family: str
    prompt: str
    signature: str
    public_tests: tuple = ()  # ((args tuple, expected stdout), ...)
    hidden_tests: tuple = ()

    @property
    def tests(self) -> tuple:
        return self.public_tests + self.hidden_tests


@dataclass(frozen=True)
class Family:
    key: str
    level: int
    signature: str
    description: str
    reference: str
    gen: Callable[[random.Random], tuple]
    edge: tuple = field(default_factory=tuple)  # argument tuples always among the hidden tests


# ------------------------------------------------------------------------------ input generators
_WORDS = ("apple", "river", "stone", "cloud", "ember", "maple", "orbit", "pixel", "quartz", "tiger", "a", "io")


def _ints(r, lo=-20, hi=50, n_lo=0, n_hi=8):
    return [r.randint(lo, hi) for _ in range(r.randint(n_lo, n_hi))]


def _sentence(r, n_lo=1, n_hi=7):
    return " ".join(r.choice(_WORDS) for _ in range(r.randint(n_lo, n_hi)))


def _expr(r):
    terms = [str(r.randint(0, 40)) for _ in range(r.randint(1, 5))]
    out = terms[0]
    for t in terms[1:]:
        out += r.choice(["+", "-"]) + t
    return out


# ------------------------------------------------------------------------------ families
F = Family
FAMILIES: list[Family] = [
    # level 1
    F("triple_minus", 1, "solve(n)", "Return 3 * n - 4.", "def solve(n):\n  return 3 * n - 4",
      lambda r: (r.randint(-50, 50),), ((0,), (-1,))),
    F("square_plus_n", 1, "solve(n)", "Return n squared plus n.", "def solve(n):\n  return n * n + n",
      lambda r: (r.randint(-30, 30),), ((0,), (1,))),
    F("last_digit", 1, "solve(n)", "Return the last digit of the non-negative integer n.",
      "def solve(n):\n  return n % 10", lambda r: (r.randint(0, 10 ** 6),), ((0,), (10,))),
    # level 2
    F("bigger", 2, "solve(a, b)", "Return the larger of a and b.",
      "def solve(a, b):\n  if a > b:\n    return a\n  return b", lambda r: (r.randint(-40, 40), r.randint(-40, 40)),
      ((5, 5), (-3, -7))),
    F("floor_mean", 2, "solve(a, b)", "Return the average of a and b rounded down.",
      "def solve(a, b):\n  return (a + b) // 2", lambda r: (r.randint(-40, 40), r.randint(-40, 40)), ((1, 2), (-1, 0))),
    F("divides", 2, "solve(a, b)", "Return True if b divides a exactly (b is never 0), else False.",
      "def solve(a, b):\n  return a % b == 0", lambda r: (r.randint(-60, 60), r.choice([1, 2, 3, 4, 5, 6, 7, -3])),
      ((0, 5), (12, -3))),
    # level 3
    F("sum_upto", 3, "solve(n)", "Return 1 + 2 + ... + n (0 when n < 1).",
      "def solve(n):\n  s = 0\n  for i in range(1, n + 1):\n    s += i\n  return s", lambda r: (r.randint(-3, 80),),
      ((0,), (1,), (-2,))),
    F("count_multiples", 3, "solve(n, m)", "Return how many of 1..n are multiples of m (m >= 1).",
      "def solve(n, m):\n  c = 0\n  for i in range(1, n + 1):\n    if i % m == 0:\n      c += 1\n  return c",
      lambda r: (r.randint(0, 100), r.randint(1, 9)), ((0, 3), (7, 7))),
    F("factorial", 3, "solve(n)", "Return n! (with 0! = 1).",
      "def solve(n):\n  f = 1\n  for i in range(2, n + 1):\n    f *= i\n  return f", lambda r: (r.randint(0, 12),),
      ((0,), (1,))),
    # level 4
    F("list_sum", 4, "solve(xs)", "Return the sum of the list xs (0 for an empty list).",
      "def solve(xs):\n  s = 0\n  for x in xs:\n    s += x\n  return s", lambda r: (_ints(r),), (([],), ([-5],))),
    F("count_even", 4, "solve(xs)", "Return how many numbers in xs are even.",
      "def solve(xs):\n  c = 0\n  for x in xs:\n    if x % 2 == 0:\n      c += 1\n  return c", lambda r: (_ints(r),),
      (([],), ([1, 3],))),
    F("list_max", 4, "solve(xs)", "Return the largest number in xs, or None for an empty list.",
      "def solve(xs):\n  if len(xs) == 0:\n    return None\n  m = xs[0]\n  for x in xs:\n    if x > m:\n      m = x\n"
      "  return m", lambda r: (_ints(r),), (([],), ([-4, -9],))),
    # level 5
    F("reverse_words", 5, "solve(s)", "Return the words of s in reverse order, joined by single spaces.",
      "def solve(s):\n  return ' '.join(reversed(s.split()))", lambda r: (_sentence(r),), (("",), ("one",))),
    F("count_vowels", 5, "solve(s)", "Return how many characters of s are vowels (a, e, i, o, u).",
      "def solve(s):\n  c = 0\n  for ch in s:\n    if ch in 'aeiou':\n      c += 1\n  return c", lambda r: (_sentence(r),),
      (("",), ("xyz",))),
    F("title_words", 5, "solve(s)", "Return s with the first letter of every word in upper case.",
      "def solve(s):\n  return ' '.join([w[0].upper() + w[1:] for w in s.split()])", lambda r: (_sentence(r),),
      (("",), ("a",))),
    # level 6
    F("fizz_list", 6, "solve(n)", "Return a list of 1..n where multiples of 3 become 'Fizz', of 5 'Buzz', of both "
      "'FizzBuzz'.",
      "def solve(n):\n  out = []\n  for i in range(1, n + 1):\n    if i % 15 == 0:\n      out.append('FizzBuzz')\n"
      "    elif i % 3 == 0:\n      out.append('Fizz')\n    elif i % 5 == 0:\n      out.append('Buzz')\n    else:\n"
      "      out.append(i)\n  return out", lambda r: (r.randint(0, 20),), ((0,), (15,))),
    F("second_largest", 6, "solve(xs)", "Return the second largest distinct value in xs, or None if there is none.",
      "def solve(xs):\n  best = None\n  second = None\n  for x in xs:\n    if best is None or x > best:\n"
      "      if best is not None:\n        second = best\n      best = x\n    elif x != best and (second is None or x > "
      "second):\n      second = x\n  return second", lambda r: (_ints(r, 0, 9),), (([],), ([4, 4, 4],), ([2, 9],))),
    F("longest_run", 6, "solve(xs)", "Return the length of the longest run of equal adjacent values in xs.",
      "def solve(xs):\n  best = 0\n  cur = 0\n  for i in range(len(xs)):\n    if i > 0 and xs[i] == xs[i - 1]:\n"
      "      cur += 1\n    else:\n      cur = 1\n    if cur > best:\n      best = cur\n  return best",
      lambda r: ([r.choice([1, 2, 3]) for _ in range(r.randint(0, 10))],), (([],), ([7],))),
    # level 7 (compositional)
    F("sum_primes", 7, "solve(n)", "Return the sum of all primes <= n.",
      "def solve(n):\n  s = 0\n  for k in range(2, n + 1):\n    ok = True\n    d = 2\n    while d * d <= k:\n"
      "      if k % d == 0:\n        ok = False\n        break\n      d += 1\n    if ok:\n      s += k\n  return s",
      lambda r: (r.randint(0, 120),), ((0,), (2,), (1,))),
    F("sorted_unique", 7, "solve(xs)", "Return the distinct values of xs in increasing order.",
      "def solve(xs):\n  out = []\n  for x in sorted(xs):\n    if len(out) == 0 or out[-1] != x:\n      out.append(x)\n"
      "  return out", lambda r: (_ints(r, -5, 5, 0, 10),), (([],), ([3, 3, 3],))),
    F("long_words", 7, "solve(s, k)", "Return how many distinct words of s are longer than k letters.",
      "def solve(s, k):\n  seen = []\n  for w in s.split():\n    if len(w) > k and w not in seen:\n      seen.append(w)\n"
      "  return len(seen)", lambda r: (_sentence(r, 0, 8), r.randint(0, 5)), (("", 2), ("apple apple", 3))),
    # level 8 (compositional)
    F("factorial_digit_sum", 8, "solve(n)", "Return the sum of the decimal digits of n!.",
      "def solve(n):\n  f = 1\n  for i in range(2, n + 1):\n    f *= i\n  s = 0\n  while f > 0:\n    s += f % 10\n"
      "    f //= 10\n  return s", lambda r: (r.randint(0, 25),), ((0,), (1,))),
    F("collatz_peak", 8, "solve(n)", "Starting from n >= 1, halve even values and map odd v to 3v + 1 until 1; "
      "return the largest value reached.",
      "def solve(n):\n  peak = n\n  while n != 1:\n    if n % 2 == 0:\n      n //= 2\n    else:\n      n = 3 * n + 1\n"
      "    if n > peak:\n      peak = n\n  return peak", lambda r: (r.randint(1, 60),), ((1,), (2,))),
    F("eval_plus_minus", 8, "solve(s)", "s is non-negative integers joined by + and - (no spaces); return its value.",
      "def solve(s):\n  total = 0\n  num = 0\n  sign = 1\n  for ch in s:\n    if ch == '+' or ch == '-':\n"
      "      total += sign * num\n      num = 0\n      sign = 1 if ch == '+' else -1\n    else:\n"
      "      num = num * 10 + int(ch)\n  return total + sign * num", lambda r: (_expr(r),), (("0",), ("7-7",))),
    # level 9 (compositional)
    F("lcm_of_list", 9, "solve(xs)", "Return the least common multiple of the positive integers in xs (1 for an "
      "empty list).",
      "def solve(xs):\n  def gcd(a, b):\n    while b:\n      a, b = b, a % b\n    return a\n  m = 1\n  for x in xs:\n"
      "    m = m * x // gcd(m, x)\n  return m", lambda r: ([r.randint(1, 12) for _ in range(r.randint(0, 5))],),
      (([],), ([7],), ([4, 6],))),
    F("mode_smallest", 9, "solve(xs)", "Return the most frequent value of xs (the smallest among ties), or None "
      "for an empty list.",
      "def solve(xs):\n  best = None\n  best_n = 0\n  for x in sorted(xs):\n    n = 0\n    for y in xs:\n"
      "      if y == x:\n        n += 1\n    if n > best_n:\n      best = x\n      best_n = n\n  return best",
      lambda r: (_ints(r, 0, 5, 0, 9),), (([],), ([2, 1, 2, 1],))),
    F("min_balance", 9, "solve(xs)", "xs are deposits (positive) and withdrawals (negative) from a balance that "
      "starts at 0; return the lowest balance reached (0 if it never drops below 0).",
      "def solve(xs):\n  b = 0\n  low = 0\n  for x in xs:\n    b += x\n    if b < low:\n      low = b\n  return low",
      lambda r: (_ints(r, -30, 30),), (([],), ([5, -2],))),
]
BY_KEY = {f.key: f for f in FAMILIES}


def families(level: int) -> list[Family]:
    return [f for f in FAMILIES if f.level == level]


# ------------------------------------------------------------------------------ tests and grading
def call_source(program: str, args: tuple) -> str:
    return f"{program}\nprint(solve({', '.join(repr(a) for a in args)}))\n"


def run_call(program: str, args: tuple, max_steps: int = GRADE_STEPS) -> micropy.ExecResult:
    return micropy.run(call_source(program, args), max_steps=max_steps)


def _expected(fam: Family, args: tuple) -> str:
    r = run_call(fam.reference, args, max_steps=10 * GRADE_STEPS)
    if not r.ok:
        raise RuntimeError(f"{fam.key}{args}: reference failed: {r.error}")
    return r.stdout


def make_problem(fam: Family, rng: random.Random, n_public: int = N_PUBLIC, n_hidden: int = N_HIDDEN) -> Problem:
    seen, args = set(), []
    edge = list(fam.edge)
    for _ in range(200):  # distinct argument tuples: public ones first, hidden ones include the edges
        if len(args) >= n_public + n_hidden:
            break
        a = edge.pop(0) if len(args) >= n_public and edge else fam.gen(rng)
        k = repr(a)
        if k not in seen:
            seen.add(k)
            args.append(a)
    tests = tuple((a, _expected(fam, a)) for a in args)
    pub, hid = tests[:n_public], tests[n_public:]
    ex = "\n".join(f"  solve({', '.join(repr(x) for x in a)}) -> {out.strip()}" for a, out in pub)
    prompt = (f"Write a Python function {fam.signature}. {fam.description}\nExamples:\n{ex}\n"
              "Write only the function, then a line with END.\n")
    pid = f"{fam.key}-{rng.getrandbits(32):08x}"
    return Problem(pid, fam.level, fam.key, prompt, fam.signature, pub, hid)


def sample_problem(rng: random.Random, level: int) -> Problem:
    return make_problem(rng.choice(families(level)), rng)


def eval_problems(level: int, n: int, seed: int = 7_000_001) -> list[Problem]:
    rng = random.Random(seed * 31 + level)
    return [sample_problem(rng, level) for _ in range(n)]


def extract_program(completion: str) -> str:
    return (completion or "").split("\nEND", 1)[0].split("END\n", 1)[0]


def grade(program: str, problem: Problem) -> dict[str, float]:
    has = bool(_SOLVE.search(program or ""))
    if not has:
        return {"has_code": 0.0, "ran_ok": 0.0, "frac_passed": 0.0, "exact": 0.0}
    ran = passed = 0
    for args, want in problem.tests:
        r = run_call(program, args)
        ran += r.ok
        passed += r.ok and r.stdout == want
    n = max(len(problem.tests), 1)
    return {"has_code": 1.0, "ran_ok": float(ran == len(problem.tests)), "frac_passed": passed / n,
            "exact": float(passed == len(problem.tests))}


def reward_of(g: dict[str, float]) -> float:
    return W_HAS_CODE * g["has_code"] + W_RAN_OK * g["ran_ok"] + W_FRAC * g["frac_passed"]


def feedback(program: str, problem: Problem, max_chars: int = 400) -> str:
    """The first public test the program fails, as the next turn's observation ('' when all pass)."""
    if not _SOLVE.search(program or ""):
        return "No function named solve was defined."
    for args, want in problem.public_tests:
        call = f"solve({', '.join(repr(a) for a in args)})"
        r = run_call(program, args)
        if not r.ok:
            return f"{call} raised {r.error}"[:max_chars]
        if r.stdout != want:
            return f"{call} returned {r.stdout.strip()}, expected {want.strip()}"[:max_chars]
    return ""


class SolveProblemEnv:
    """``sample(level)``, ``held_out(level, n)`` and ``reward(completion, problem)``: the environment
    interface of ``rl.curriculum.CurriculumTaskSource``."""

    num_levels = NUM_LEVELS

    def __init__(self, seed: int = 0):
        self.rng = random.Random(seed)

    def sample(self, level: int) -> Problem:
        return sample_problem(self.rng, level)

    def held_out(self, level: int, n: int, seed: int = 7_000_001) -> list[Problem]:
        return eval_problems(level, n, seed)

    @staticmethod
    def reward(completion: str, problem: Problem) -> float:
        return reward_of(grade(extract_program(completion), problem))

    @staticmethod
    def solved(completion: str, problem: Problem) -> bool:
        return grade(extract_program(completion), problem)["exact"] == 1.0
