"""The sandboxed Python-subset interpreter: language cases (program -> stdout), errors (program ->
error kind), limits and determinism."""

import pytest

from marin_experiments_b200.rl.micropy import run

OK = [
    ("print(2)", "2\n"), ("print('hi')", "hi\n"), ("print(True, False, None)", "True False None\n"),
    ("print(1 + 2 * 3)", "7\n"), ("print((1 + 2) * 3)", "9\n"), ("print(7 - 3 - 1)", "3\n"),
    ("print(7 // 2, 7 % 3, 2 ** 10, -7 // 2)", "3 1 1024 -4\n"), ("print(7 / 2, 6 / 3)", "3.5 2.0\n"),
    ("print(0.1 + 0.2)", f"{0.1 + 0.2}\n"), ("print(-2 ** 2, 2 ** 3 ** 2)", "-4 512\n"),
    ("print(-5, +5, not True, not 0)", "-5 5 False True\n"),
    ("x = 5\ny = x + 1\nprint(y)", "6\n"), ("x = 1\nx += 4\nx *= 2\nprint(x)", "10\n"),
    ("x = 10\nx -= 3\nx //= 2\nprint(x)", "3\n"), ("a, b = 1, 2\na, b = b, a\nprint(a, b)", "2 1\n"),
    ("x = y = 5\nprint(x, y)", "5 5\n"), ("xs = [1, 2, 3]\nxs[0] = 9\nprint(xs)", "[9, 2, 3]\n"),
    ("xs = [1, 2]\nxs[1] += 5\nprint(xs)", "[1, 7]\n"),
    ("print(1 < 2 < 3, 1 < 2 > 5, 1 == 1, 1 != 2)", "True False True True\n"),
    ("print(True and 'yes', False or 'no', 0 and 1, 1 or 2)", "yes no 0 1\n"),
    ("print(3 in [1, 2, 3], 'a' not in 'xyz')", "True True\n"),
    ("x = 5\nprint('big' if x > 3 else 'small')", "big\n"),
    ("x = 2\nif x == 1:\n  print('a')\nelif x == 2:\n  print('b')\nelse:\n  print('c')", "b\n"),
    ("i = 0\nwhile i < 3:\n  print(i)\n  i += 1", "0\n1\n2\n"),
    ("i = 0\nwhile True:\n  if i == 2:\n    break\n  print(i)\n  i += 1", "0\n1\n"),
    ("i = 0\nwhile i < 5:\n  i += 1\n  if i % 2 == 0:\n    continue\n  print(i)", "1\n3\n5\n"),
    ("for i in range(1, 6, 2):\n  print(i)", "1\n3\n5\n"), ("for c in 'ab':\n  print(c)", "a\nb\n"),
    ("for i in range(3):\n  print(i)\nelse:\n  print('done')", "0\n1\n2\ndone\n"),
    ("for i in range(3):\n  if i == 1:\n    break\nelse:\n  print('done')\nprint('after')", "after\n"),
    ("def add(a, b):\n  return a + b\nprint(add(2, 3))", "5\n"),
    ("def g(n, s='hi'):\n  return s + ' ' + n\nprint(g('x'))\nprint(g('y', 'yo'))", "hi x\nyo y\n"),
    ("def f(a, b):\n  return a - b\nprint(f(b=1, a=10))", "9\n"),
    ("def f():\n  x = 99\n  return x\nx = 1\nprint(f())\nprint(x)", "99\n1\n"),
    ("G = 7\ndef f():\n  return G + 1\nprint(f())", "8\n"),
    ("def fib(n):\n  if n < 2:\n    return n\n  return fib(n - 1) + fib(n - 2)\nprint(fib(10))", "55\n"),
    ("def f():\n  pass\nprint(f())", "None\n"),
    ("print([x * x for x in range(5)])", "[0, 1, 4, 9, 16]\n"),
    ("print([x for x in range(10) if x % 2 == 0])", "[0, 2, 4, 6, 8]\n"),
    ("print([(a, b) for a in range(2) for b in 'xy'])", "[(0, 'x'), (0, 'y'), (1, 'x'), (1, 'y')]\n"),
    ("xs = [1, 2, 3, 4]\nprint(xs[0], xs[-1], xs[1:3], xs[::-1])", "1 4 [2, 3] [4, 3, 2, 1]\n"),
    ("print([1, 2] + [3], [0] * 3)", "[1, 2, 3] [0, 0, 0]\n"),
    ("xs = [1, 2]\nxs.append(3)\nxs.insert(0, 0)\nprint(xs)\nprint(xs.pop())\nprint(xs.index(2), xs.count(1))",
     "[0, 1, 2, 3]\n3\n2 1\n"),
    ("print(len([1, 2, 3]), sum([1, 2, 3]), min([3, 1, 2]), max(3, 1, 2))", "3 6 1 3\n"),
    ("print(sorted([3, 1, 2]), reversed([1, 2, 3]), list(range(3)))", "[1, 2, 3] [3, 2, 1] [0, 1, 2]\n"),
    ("print(enumerate(['a', 'b']), zip([1, 2], [3, 4]))", "[(0, 'a'), (1, 'b')] [(1, 3), (2, 4)]\n"),
    ("s = 'hello'\nprint(s[0], s[-1], s[1:4])", "h o ell\n"),
    ("print('ab' + 'cd', 'ab' * 3, 'b' in 'abc')", "abcd ababab True\n"),
    ("print('Hi'.upper(), 'Hi'.lower(), '  x '.strip(), 'a,b,c'.split(','))", "HI hi x ['a', 'b', 'c']\n"),
    ("print('-'.join(['a', 'b']), 'abc'.replace('b', 'X'), 'abc'.find('c'))", "a-b aXc 2\n"),
    ("x = 7\nprint(f'x is {x}', f'{2 + 3}', f'{3.14159:.2f}', f'{42:05d}')", "x is 7 5 3.14 00042\n"),
    ("print('%d-%s' % (3, 'x'), '%.1f' % 2.5)", "3-x 2.5\n"),
    ("print(1, 2, 3, sep='-')", "1-2-3\n"), ("print('a', end='')\nprint('b')", "ab\n"),
    ("print('a', 'b', sep='|', end='!')", "a|b!"), ("print()", "\n"),
    ("for i in range(1, 6):\n  if i % 15 == 0:\n    print('FizzBuzz')\n  elif i % 3 == 0:\n    print('Fizz')\n"
     "  elif i % 5 == 0:\n    print('Buzz')\n  else:\n    print(i)", "1\n2\nFizz\n4\nBuzz\n"),
    ("print(int('12') + 1, str(5) + '!', float('2.5'), abs(-3), round(2.675, 2), divmod(7, 2))",
     "13 5! 2.5 3 2.67 (3, 1)\n"),
]

ERR = [
    ("print(", "SyntaxError:"), ("print(undefined_var)", "NameError:"), ("print(1 / 0)", "ZeroDivisionError:"),
    ("print(1 // 0)", "ZeroDivisionError:"), ("print(1 % 0)", "ZeroDivisionError:"),
    ("xs = [1, 2]\nprint(xs[5])", "IndexError:"), ("s = 'ab'\nprint(s[9])", "IndexError:"),
    ("print('a' + 1)", "TypeError:"), ("x = 5\nprint(x())", "TypeError:"), ("a, b = 1, 2, 3", "ValueError:"),
    ("ys = [i for i in range(3)]\nprint(i)", "NameError:"),
    ("import os", "UnsupportedSyntax: Import"), ("from os import getcwd", "UnsupportedSyntax: ImportFrom"),
    ("class Foo:\n  pass", "UnsupportedSyntax: ClassDef"), ("with open('x') as f:\n  pass", "UnsupportedSyntax: With"),
    ("try:\n  pass\nexcept:\n  pass", "UnsupportedSyntax: Try"), ("f = lambda x: x", "UnsupportedSyntax: Lambda"),
    ("def f():\n  global x\n  x = 1\nf()", "UnsupportedSyntax: Global"),
    ("print(sum(x for x in range(3)))", "UnsupportedSyntax:"), ("@deco\ndef f():\n  pass", "UnsupportedSyntax: decorators"),
    ("print({'a': 1})", "UnsupportedSyntax: Dict"), ("print({1, 2})", "UnsupportedSyntax: Set"),
    ("assert False", "UnsupportedSyntax: Assert"), ("x = 1\ndel x", "UnsupportedSyntax: Delete"),
    ("yield 1", "UnsupportedSyntax: Yield"), ("print(*[1, 2])", "UnsupportedSyntax:"),
    ("eval('1+1')", "NameError:"), ("exec('x=1')", "NameError:"), ("open('f')", "NameError:"), ("input()", "NameError:"),
    ("print((1).__class__)", "AttributeError:"), ("print([].__class__.__bases__)", "AttributeError:"),
    ("x = 5\nprint(x.real)", "AttributeError:"), ("print('abc'.__len__())", "AttributeError:"),
    ("[].sort()", "AttributeError:"), ("'x'.format()", "AttributeError:"),
    ("print(2 ** 100000)", "OverflowError:"),
] + [(f"{n}()", "NameError:") for n in ("__import__", "globals", "locals", "vars", "getattr", "setattr", "type")]


@pytest.mark.parametrize("src,want", OK)
def test_programs(src, want):
    r = run(src)
    assert r.ok and r.error is None, r.error
    assert r.stdout == want


@pytest.mark.parametrize("src,prefix", ERR)
def test_errors(src, prefix):
    r = run(src)
    assert not r.ok and r.error is not None and r.error.startswith(prefix), r.error


def test_step_limit():
    r = run("while True:\n  pass", max_steps=1000)
    assert not r.ok and r.error == "StepLimit: exceeded max_steps" and r.steps >= 1000
    r = run("def f():\n  return f()\nf()", max_steps=5000)
    assert not r.ok and r.error in ("StepLimit: exceeded max_steps", "RecursionError: maximum recursion depth exceeded")


def test_output_limit_keeps_prefix():
    r = run("while True:\n  print('x')", max_output=10)
    assert not r.ok and r.error == "OutputLimit: exceeded max_output" and len(r.stdout) == 10
    r = run("print('hello world')", max_output=5)
    assert r.error == "OutputLimit: exceeded max_output" and r.stdout == "hello"


def test_deterministic():
    src = "def fib(n):\n  return n if n < 2 else fib(n - 1) + fib(n - 2)\nprint(fib(12))"
    assert run(src) == run(src)


_AGREE = [
    "print(7, 'a', True, None)",
    "print(17 // 5, -17 // 5, 17 % 5, -17 % 5, 2 ** 10, 7 / 2)",
    "print(0.1 + 0.2, 3.5 * 2, round(2.675, 2), -2 ** 2)",
    "print(not 0, -(-3), +4, ~5)",
    "a, b = 1, 2\na, b = b, a\nprint(a, b)",
    "x = [1, 2, 3]\nx[1] = 9\nx[-1] += 1\nprint(x)",
    "print(1 < 2 < 3, 3 > 2 > 2, 1 == 1.0, 'a' < 'b')",
    "print(0 or 'x', 1 and 0, [] or [1], 2 in [1, 2], 'bc' in 'abc', 3 not in (1, 2))",
    "print('y' if 2 > 1 else 'n')",
    "n = 0\nwhile True:\n  n += 1\n  if n % 2:\n    continue\n  if n > 6:\n    break\nprint(n)",
    "for i in range(3):\n  pass\nelse:\n  print('done', i)",
    "for i in range(5):\n  if i == 2:\n    break\nelse:\n  print('no')\nprint(i)",
    "def f(a, b=2, c=3):\n  return a + b * c\nprint(f(1), f(1, c=10), f(b=0, a=5))",
    "g = 5\ndef h():\n  x = g + 1\n  return x\nprint(h())",
    "def fib(n):\n  return n if n < 2 else fib(n - 1) + fib(n - 2)\nprint(fib(15))",
    "def nothing():\n  pass\nprint(nothing())",
    "print([i * i for i in range(6) if i % 2])",
    "xs = list(range(10))\nprint(xs[2:8:2], xs[::-3], xs[-2:], len(xs))",
    "print([1, 2] + [3] * 2, 'ab' * 3)",
    "x = [3, 1, 2]\nx.append(5)\nx = sorted(x)\nx.insert(0, 9)\nprint(x, x.pop(), x.index(3), x.count(9))",
    "print(sum([1, 2, 3]), min(4, 2, 8), max([1, 9, 3]), sorted([3, 1, 2], reverse=True), abs(-4))",
    "print(list(enumerate('ab', 1)), list(zip([1, 2], 'xy')), list(reversed([1, 2, 3])))",
    "s = 'Hello World'\nprint(s.lower(), s.upper(), s.split(), s.replace('l', 'L'), s.startswith('He'), s.find('o'))",
    "print(' x '.strip(), ','.join(['a', 'b']), 'abc'[1], 'abc'[::-1], 'a-b-c'.split('-'))",
    "v = 3.14159\nn = 42\nprint(f'{n:5d}|{v:.2f}|{n * 2}|{\"q\"}')",
    "print('%d items at %.1f %s' % (3, 2.25, 'each'))",
    "print(1, 2, sep='-', end='!\\n')\nprint()\nprint('a', 'b', sep='')",
    "print(int('12') + int(3.9), float('2.5'), str(7) + '!', bool(''), divmod(17, 5))",
]


@pytest.mark.parametrize("src", _AGREE)
def test_agrees_with_cpython(src):
    import contextlib
    import io

    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        exec(compile(src, "<p>", "exec"), {})  # the programs above, written in this file
    r = run(src)
    assert r.ok, r.error
    assert r.stdout == buf.getvalue()


@pytest.mark.parametrize("src,kind", [
    ("print(1 +", "SyntaxError"), ("print(zz)", "NameError"), ("print(1 / 0)", "ZeroDivisionError"),
    ("print([1][3])", "IndexError"), ("print(1 + 'a')", "TypeError"), ("x = 3\nx()", "TypeError"),
    ("a, b = [1, 2, 3]", "ValueError"), ("while True:\n  pass", "StepLimit"),
    ("def f():\n  return f()\nf()", "RecursionError"), ("import os", "UnsupportedSyntax"),
    ("from os import path", "UnsupportedSyntax"), ("class A:\n  pass", "UnsupportedSyntax"),
    ("with open('x') as f:\n  pass", "UnsupportedSyntax"),
    ("[].sort()", "AttributeError"),  # in-place sort is outside the whitelisted list methods
    ("def f(*a):\n  return a", "UnsupportedSyntax"),
])
def test_error_kinds(src, kind):
    r = run(src, max_steps=20_000)
    assert not r.ok and r.error.startswith(kind), r.error
