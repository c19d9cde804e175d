"""Tiered, parameterised coding tasks for single-turn program-writing RL, a held-out evaluation
ladder and the transcript format shared by SFT and RL (tunix-delphi-rl/environments/coding_env.py:1-1173,
tunix-delphi-rl/problems/coding_tasks.py:1-1001, tunix-delphi-rl/training/train_coding.py:1-326).

The policy sees ``CODE_FEWSHOT`` + ``Task: <prompt>`` and writes a program ended by a line ``END``;
the sandboxed interpreter (``rl.micropy``) runs it and the reward compares its stdout with the
gold, which is what the family's reference solution prints. Every family draws fresh parameters
per sample, so the gold changes from sample to sample and printing a constant cannot win a group:
the policy has to write a program that computes.

Tiers (``FAMILIES[t]``):

* 0 -- print a literal (integer, word, float, boolean, upper-case phrase);
* 1 -- one operation on given operands (``+ - *``, floor division, modulo, power, a parenthesised
  expression, true division);
* 2 -- variables and branches (larger of two, absolute difference, parity word, sign word, letter
  grade, swap, clamp);
* 3 -- loops over ranges and strings (sum of a range, countdown, product, sum of multiples, vowel
  count, reversed word, joined range, list maximum, character count);
* 4 -- functions and recursion (Fibonacci, greatest common divisor, primality, digit sum, Collatz
  steps, power by repeated multiplication, triangular numbers);
* 5 -- small algorithms (sorting, second largest, digital root, n-th prime, palindrome test,
  base-2 digits, run-length encoding).

``eval_tasks()`` is a fixed ladder drawn from seeds no training sampler uses; ``evaluate(generate,
tasks)`` reports the greedy solve rate per tier. ``code_reward`` is dense (has code 0.1, ran 0.3,
output similarity 0.6, exact 1.0, as in ``rl.code_agent``), so a group has a signal before any
sample is exact. ``CodeTaskEnv`` is the ``sample`` / ``reward`` interface of ``rl.learner``.
"""

from __future__ import annotations

import random
from collections.abc import Callable
from dataclasses import dataclass

from . import micropy
from .code_agent import grade, round_reward
from .envs import Task

GRADE_STEPS = 50_000
EVAL_STEPS = 400_000

CODE_FEWSHOT = (
    "Write a short Python program for each task. End the program with a line containing only END.\n"
    "Task: Print the number 7.\n"
    "print(7)\n"
    "END\n"
    "Task: Print 12 times 9.\n"
    "print(12 * 9)\n"
    "END\n"
    "Task: Print the numbers from 1 to 3, one per line.\n"
    "for i in range(1, 4):\n"
    "  print(i)\n"
    "END\n"
)

_STOPS = ("\nEND", "\nTask:", "\n\n\n")


@dataclass(frozen=True)
class CodeTask:
    tier: int
    family: str
    prompt: str
    solution: str
    gold: str


def build_prompt(task_prompt: str) -> str:
    return f"{CODE_FEWSHOT}Task: {task_prompt}\n"


def extract_program(completion: str) -> str:
    """The completion up to the ``END`` line or a new ``Task:`` (whichever comes first)."""
    text = "\n" + (completion or "")
    cut = min((text.find(s) for s in _STOPS if text.find(s) >= 0), default=len(text))
    return text[1:cut] if cut > 0 else ""


# ---------------------------------------------------------------------------------- families
_WORDS = ("lattice", "photon", "quiver", "meadow", "cobalt", "harbor", "ember", "zephyr", "tundra", "violet")
_PALS = ("level", "rotor", "civic", "radar", "refer", "stats", "kayak")


def _t0_int(r):
    v = r.randint(-999, 999)
    return f"Print the number {v}.", f"print({v})"


def _t0_word(r):
    w = r.choice(_WORDS)
    return f"Print the word {w}.", f"print('{w}')"


def _t0_float(r):
    v = round(r.uniform(0.1, 99.9), 1)
    return f"Print the decimal number {v}.", f"print({v})"


def _t0_bool(r):
    b = r.choice(["True", "False"])
    return f"Print the boolean value {b}.", f"print({b})"


def _t0_upper(r):
    w = r.choice(_WORDS)
    return f"Print the word {w} in capital letters.", f"print('{w.upper()}')"


def _t1_arith(r):
    a, b = r.randint(2, 99), r.randint(2, 99)
    op, word = r.choice([("+", "plus"), ("-", "minus"), ("*", "times")])
    return f"Print {a} {word} {b}.", f"print({a} {op} {b})"


def _t1_floordiv(r):
    a, b = r.randint(20, 500), r.randint(2, 19)
    return f"Print {a} divided by {b}, rounded down to a whole number.", f"print({a} // {b})"


def _t1_mod(r):
    a, b = r.randint(20, 500), r.randint(2, 19)
    return f"Print the remainder when {a} is divided by {b}.", f"print({a} % {b})"


def _t1_pow(r):
    a, b = r.randint(2, 9), r.randint(2, 6)
    return f"Print {a} raised to the power {b}.", f"print({a} ** {b})"


def _t1_parens(r):
    a, b, c = r.randint(2, 30), r.randint(2, 30), r.randint(2, 9)
    return f"Print the sum of {a} and {b}, multiplied by {c}.", f"print(({a} + {b}) * {c})"


def _t1_truediv(r):
    b = r.choice([2, 4, 5, 8, 10])
    a = r.randint(1, 99)
    return f"Print {a} divided by {b} as a decimal number.", f"print({a} / {b})"


def _t2_max(r):
    a, b = r.sample(range(-50, 100), 2)
    return (f"Set a = {a} and b = {b}, then print the larger of the two using an if statement.",
            f"a = {a}\nb = {b}\nif a > b:\n  print(a)\nelse:\n  print(b)")


def _t2_absdiff(r):
    a, b = r.randint(-50, 99), r.randint(-50, 99)
    return (f"Print the absolute difference between {a} and {b}.",
            f"d = {a} - {b}\nif d < 0:\n  d = -d\nprint(d)")


def _t2_parity(r):
    n = r.randint(0, 999)
    return (f"Print even if {n} is even, otherwise print odd.",
            f"n = {n}\nif n % 2 == 0:\n  print('even')\nelse:\n  print('odd')")


def _t2_sign(r):
    n = r.choice([0, r.randint(-99, -1), r.randint(1, 99)])
    return (f"Print positive, negative or zero according to the sign of {n}.",
            f"n = {n}\nif n > 0:\n  print('positive')\nelif n < 0:\n  print('negative')\nelse:\n  print('zero')")


def _t2_grade(r):
    s = r.randint(0, 100)
    return (f"A score of {s} gets A from 90, B from 80, C from 70 and F below 70. Print the letter.",
            f"s = {s}\nif s >= 90:\n  print('A')\nelif s >= 80:\n  print('B')\nelif s >= 70:\n  print('C')\n"
            "else:\n  print('F')")


def _t2_swap(r):
    a, b = r.randint(1, 99), r.randint(1, 99)
    return (f"Set x = {a} and y = {b}, swap them, then print x and y separated by a space.",
            f"x = {a}\ny = {b}\nx, y = y, x\nprint(x, y)")


def _t2_clamp(r):
    lo, hi = sorted(r.sample(range(0, 100), 2))
    v = r.randint(-20, 120)
    return (f"Print {v} limited to the range from {lo} to {hi}.",
            f"v = {v}\nif v < {lo}:\n  v = {lo}\nif v > {hi}:\n  v = {hi}\nprint(v)")


def _t3_sum_range(r):
    a = r.randint(1, 20)
    b = a + r.randint(3, 60)
    return (f"Print the sum of the integers from {a} to {b} using a loop.",
            f"s = 0\nfor i in range({a}, {b + 1}):\n  s += i\nprint(s)")


def _t3_countdown(r):
    n = r.randint(3, 9)
    return (f"Print the numbers from {n} down to 1, one per line.",
            f"i = {n}\nwhile i >= 1:\n  print(i)\n  i -= 1")


def _t3_product(r):
    a = r.randint(1, 5)
    b = a + r.randint(2, 6)
    return (f"Print the product of the integers from {a} to {b}.",
            f"p = 1\nfor i in range({a}, {b + 1}):\n  p *= i\nprint(p)")


def _t3_multiples(r):
    m, n = r.randint(2, 9), r.randint(20, 200)
    return (f"Print the sum of all multiples of {m} below {n}.",
            f"s = 0\nfor i in range({n}):\n  if i % {m} == 0:\n    s += i\nprint(s)")


def _t3_vowels(r):
    w = r.choice(_WORDS) + r.choice(_WORDS)
    return (f"Print how many vowels (a, e, i, o, u) the word {w} has.",
            f"c = 0\nfor ch in '{w}':\n  if ch in 'aeiou':\n    c += 1\nprint(c)")


def _t3_reverse(r):
    w = r.choice(_WORDS)
    return f"Print the word {w} backwards.", f"print('{w}'[::-1])"


def _t3_join(r):
    a = r.randint(0, 10)
    b = a + r.randint(2, 8)
    sep = r.choice(["-", ",", "+"])
    return (f"Print the numbers from {a} to {b} joined by '{sep}'.",
            f"print('{sep}'.join([str(i) for i in range({a}, {b + 1})]))")


def _t3_listmax(r):
    xs = [r.randint(-50, 200) for _ in range(r.randint(4, 8))]
    return (f"Find the largest number in the list {xs} with a loop and print it.",
            f"xs = {xs}\nm = xs[0]\nfor x in xs:\n  if x > m:\n    m = x\nprint(m)")


def _t3_charcount(r):
    w = r.choice(_WORDS) * 2
    ch = r.choice(sorted(set(w)))
    return (f"Print how many times the letter {ch} appears in {w}.",
            f"c = 0\nfor x in '{w}':\n  if x == '{ch}':\n    c += 1\nprint(c)")


def _t4_fib(r):
    n = r.randint(5, 20)
    return (f"Write a function fib(n) with fib(0) = 0 and fib(1) = 1 and print fib({n}).",
            f"def fib(n):\n  a, b = 0, 1\n  for i in range(n):\n    a, b = b, a + b\n  return a\nprint(fib({n}))")


def _t4_gcd(r):
    g = r.randint(2, 12)
    a, b = g * r.randint(2, 30), g * r.randint(2, 30)
    return (f"Write a function gcd(a, b) and print the greatest common divisor of {a} and {b}.",
            f"def gcd(a, b):\n  while b:\n    a, b = b, a % b\n  return a\nprint(gcd({a}, {b}))")


def _t4_prime(r):
    n = r.randint(20, 300)
    return (f"Write a function is_prime(n) and print whether {n} is prime (True or False).",
            f"def is_prime(n):\n  if n < 2:\n    return False\n  d = 2\n  while d * d <= n:\n    if n % d == 0:\n"
            f"      return False\n    d += 1\n  return True\nprint(is_prime({n}))")


def _t4_digitsum(r):
    n = r.randint(100, 999999)
    return (f"Write a function that returns the sum of the digits of a number and print it for {n}.",
            f"def digit_sum(n):\n  s = 0\n  while n > 0:\n    s += n % 10\n    n //= 10\n  return s\n"
            f"print(digit_sum({n}))")


def _t4_collatz(r):
    n = r.randint(3, 60)
    return (f"Starting from {n}, repeatedly halve even numbers and map odd n to 3n + 1. Print how many steps "
            "it takes to reach 1.",
            f"n = {n}\nc = 0\nwhile n != 1:\n  if n % 2 == 0:\n    n //= 2\n  else:\n    n = 3 * n + 1\n  c += 1\n"
            "print(c)")


def _t4_power(r):
    a, b = r.randint(2, 7), r.randint(2, 8)
    return (f"Write a recursive function power(a, b) that multiplies a by itself b times and print power({a}, {b}).",
            f"def power(a, b):\n  if b == 0:\n    return 1\n  return a * power(a, b - 1)\nprint(power({a}, {b}))")


def _t4_triangular(r):
    n = r.randint(3, 12)
    return (f"Write a function tri(k) returning 1 + 2 + ... + k and print tri(1) to tri({n}) separated by spaces.",
            f"def tri(k):\n  return k * (k + 1) // 2\nprint(' '.join([str(tri(i)) for i in range(1, {n + 1})]))")


def _t5_sort(r):
    xs = [r.randint(-30, 99) for _ in range(r.randint(5, 8))]
    return (f"Sort the list {xs} in increasing order without using sorted and print it.",
            f"xs = {xs}\nn = len(xs)\nfor i in range(n):\n  for j in range(n - 1 - i):\n    if xs[j] > xs[j + 1]:\n"
            "      xs[j], xs[j + 1] = xs[j + 1], xs[j]\nprint(xs)")


def _t5_second(r):
    xs = r.sample(range(-40, 150), r.randint(5, 8))
    return (f"Print the second largest number in the list {xs}.",
            f"xs = {xs}\nbest = max(xs)\nsecond = min(xs)\nfor x in xs:\n  if x != best and x > second:\n"
            "    second = x\nprint(second)")


def _t5_droot(r):
    n = r.randint(10, 10 ** 7)
    return (f"Repeatedly replace {n} by the sum of its digits until one digit is left, then print it.",
            f"n = {n}\nwhile n >= 10:\n  s = 0\n  while n > 0:\n    s += n % 10\n    n //= 10\n  n = s\nprint(n)")


def _t5_nthprime(r):
    k = r.randint(3, 40)
    return (f"Print the {k}-th prime number (the 1st is 2).",
            f"count = 0\nn = 1\nwhile count < {k}:\n  n += 1\n  ok = True\n  d = 2\n  while d * d <= n:\n"
            f"    if n % d == 0:\n      ok = False\n      break\n    d += 1\n  if ok:\n    count += 1\nprint(n)")


def _t5_palindrome(r):
    w = r.choice(_PALS) if r.random() < 0.5 else r.choice(_WORDS)
    return (f"Print yes if {w} reads the same backwards, otherwise print no.",
            f"w = '{w}'\nok = True\nfor i in range(len(w) // 2):\n  if w[i] != w[len(w) - 1 - i]:\n    ok = False\n"
            "print('yes' if ok else 'no')")


def _t5_binary(r):
    n = r.randint(2, 4000)
    return (f"Print {n} written in base 2 (digits only).",
            f"n = {n}\nd = ''\nwhile n > 0:\n  d = str(n % 2) + d\n  n //= 2\nprint(d)")


def _t5_rle(r):
    s = "".join(r.choice("ab") * r.randint(1, 4) for _ in range(r.randint(3, 6)))
    return (f"Run-length encode {s}: for each run print the letter followed by its length, all on one line.",
            f"s = '{s}'\nout = ''\ni = 0\nwhile i < len(s):\n  j = i\n  while j < len(s) and s[j] == s[i]:\n"
            "    j += 1\n  out += s[i] + str(j - i)\n  i = j\nprint(out)")


FAMILIES: dict[int, list[Callable]] = {
    0: [_t0_int, _t0_word, _t0_float, _t0_bool, _t0_upper],
    1: [_t1_arith, _t1_floordiv, _t1_mod, _t1_pow, _t1_parens, _t1_truediv],
    2: [_t2_max, _t2_absdiff, _t2_parity, _t2_sign, _t2_grade, _t2_swap, _t2_clamp],
    3: [_t3_sum_range, _t3_countdown, _t3_product, _t3_multiples, _t3_vowels, _t3_reverse, _t3_join, _t3_listmax,
        _t3_charcount],
    4: [_t4_fib, _t4_gcd, _t4_prime, _t4_digitsum, _t4_collatz, _t4_power, _t4_triangular],
    5: [_t5_sort, _t5_second, _t5_droot, _t5_nthprime, _t5_palindrome, _t5_binary, _t5_rle],
}
TIERS = tuple(sorted(FAMILIES))


def make_task(rng: random.Random, tier: int, family: Callable | None = None) -> CodeTask:
    fam = family or rng.choice(FAMILIES[tier])
    prompt, sol = fam(rng)
    res = micropy.run(sol, max_steps=EVAL_STEPS)
    if not res.ok:
        raise RuntimeError(f"{fam.__name__}: reference solution failed: {res.error}\n{sol}")
    return CodeTask(tier, fam.__name__.lstrip("_"), prompt, sol, res.stdout)


def sample_tasks(n: int, seed: int, tiers: tuple[int, ...] = TIERS) -> list[CodeTask]:
    rng = random.Random(seed)
    return [make_task(rng, rng.choice(tiers)) for _ in range(n)]


def eval_tasks(per_family: int = 1, seed: int = 2_000_003) -> list[CodeTask]:
    """The held-out ladder: ``per_family`` tasks of every family, tier by tier, from a seed that the
    training samplers do not use."""
    rng = random.Random(seed)
    return [make_task(rng, t, fam) for t in TIERS for fam in FAMILIES[t] for _ in range(per_family)]


def code_reward(completion: str, gold: str, max_steps: int = GRADE_STEPS) -> float:
    prog = extract_program(completion)
    res = micropy.run(prog, max_steps=max_steps) if prog.strip() else micropy.ExecResult("", False, "no program", 0)
    return round_reward(grade(res, prog, gold))


def code_metrics(completions: list[str], golds: list[str]) -> dict[str, float]:
    n = max(len(completions), 1)
    has = ran = exact = 0
    for c, g in zip(completions, golds):
        prog = extract_program(c)
        if not prog.strip():
            continue
        has += 1
        res = micropy.run(prog, max_steps=GRADE_STEPS)
        ran += res.ok
        exact += res.ok and res.stdout == g
    return {"code/has_code": has / n, "code/ran_ok": ran / n, "code/solve_ratio": exact / n}


def sft_segments(task: CodeTask) -> list[tuple[str, int]]:
    """The SFT transcript in the RL prompt format: prompt as context (0), program + END trained (1)."""
    return [(build_prompt(task.prompt), 0), (f"{task.solution}\nEND\n", 1)]


class CodeTaskEnv:
    """``sample`` / ``reward`` for ``rl.learner.GRPOLearner``; the gold rides in the task's answer."""

    def __init__(self, seed: int = 0, tiers: tuple[int, ...] = TIERS):
        self.rng, self.tiers = random.Random(seed), tuple(tiers)

    def sample(self) -> Task:
        t = make_task(self.rng, self.rng.choice(self.tiers))
        return Task(build_prompt(t.prompt), t.gold)

    @staticmethod
    def reward(completion: str, answer: str) -> float:
        return code_reward(completion, answer)


def evaluate(generate: Callable[[str], str], tasks: list[CodeTask]) -> dict:
    """Greedy solve rate per tier and overall; ``generate(prompt) -> completion``."""
    per: dict[int, list[int]] = {}
    for t in tasks:
        prog = extract_program(generate(build_prompt(t.prompt)))
        res = micropy.run(prog, max_steps=EVAL_STEPS)
        per.setdefault(t.tier, []).append(int(res.ok and res.stdout == t.gold))
    out = {f"tier{k}": sum(v) / len(v) for k, v in sorted(per.items())}
    out["solved"] = sum(sum(v) for v in per.values())
    out["total"] = sum(len(v) for v in per.values())
    return out
