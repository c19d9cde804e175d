"""A sandboxed, deterministic interpreter for a small subset of Python: the executor and verifier
of the agentic-coding RL environments (tunix-delphi-rl/environments/micropython.py describes the
same contract; this is an independent implementation of it).

``run(source)`` parses the program with ``ast`` and evaluates the tree itself -- never ``exec`` or
``eval`` -- and returns ``ExecResult(stdout, ok, error, steps)``:

* deterministic: no clock, randomness, imports, files or host state; the same source always
  gives the same result, step count included;
* contained: only whitelisted builtins (``print len range int str float bool abs min max sum
  sorted reversed enumerate zip list round divmod``) and whitelisted methods of ``str`` and
  ``list``; no attribute access other than those method calls, nothing with a leading underscore;
* bounded: every evaluated node costs a step (``max_steps``), printed text is capped
  (``max_output``; the prefix that fit is kept), and calls nest at most ``max_depth`` deep, so
  infinite loops and runaway recursion end with ``ok=False``.

Errors never propagate: they come back as ``"Kind: message"`` -- Python's own exception names for
program errors (``NameError``, ``TypeError``, ``ZeroDivisionError``, ...), ``SyntaxError`` for
unparsable source, ``UnsupportedSyntax: <node>`` for constructs outside the subset (imports,
classes, try/with, lambda, global, generators, decorators, dict / set literals, assert / del /
yield, starred arguments), ``StepLimit: exceeded max_steps`` and ``OutputLimit: exceeded
max_output``.

Supported: int / float / str / bool / None constants, lists and tuples, arithmetic (Python
semantics, floor division and modulo included, ``%`` string formatting), comparisons (chained),
``and`` / ``or`` / ``not``, ``in``, conditional expressions, subscripts and slices, list
comprehensions (own scope), f-strings with format specs, assignment (targets: names, tuples,
subscripts), augmented assignment, ``if`` / ``while`` / ``for`` (with ``else``), ``break`` /
``continue``, ``def`` with defaults and keyword arguments, ``return``, recursion.
"""

from __future__ import annotations

import ast
import dataclasses
import operator


@dataclasses.dataclass(frozen=True)
class ExecResult:
    stdout: str
    ok: bool
    error: str | None
    steps: int


class _Fail(Exception):
    """A program error reported as ``kind: message``."""

    def __init__(self, kind: str, msg: str):
        super().__init__(f"{kind}: {msg}")
        self.text = f"{kind}: {msg}"


class _Stop(Exception):
    """A limit was hit (steps / output)."""

    def __init__(self, text: str):
        super().__init__(text)
        self.text = text


class _Break(Exception):
    pass


class _Continue(Exception):
    pass


class _Return(Exception):
    def __init__(self, value):
        super().__init__()
        self.value = value


class _UserFn:
    def __init__(self, node: ast.FunctionDef, defaults: list, globals_: dict):
        self.node, self.defaults, self.globals = node, defaults, globals_
        self.name = node.name


# statement / expression node types outside the subset, by the name reported
_UNSUPPORTED = {
    ast.Import: "Import", ast.ImportFrom: "ImportFrom", ast.ClassDef: "ClassDef", ast.With: "With",
    ast.Try: "Try", ast.Lambda: "Lambda", ast.Global: "Global", ast.Nonlocal: "Nonlocal",
    ast.GeneratorExp: "GeneratorExp", ast.Dict: "Dict", ast.Set: "Set", ast.DictComp: "DictComp",
    ast.SetComp: "SetComp", ast.Assert: "Assert", ast.Delete: "Delete", ast.Yield: "Yield",
    ast.YieldFrom: "YieldFrom", ast.Await: "Await", ast.AsyncFunctionDef: "AsyncFunctionDef",
    ast.Raise: "Raise", ast.Starred: "Starred", ast.NamedExpr: "NamedExpr", ast.Match: "Match",
}
if hasattr(ast, "TryStar"):
    _UNSUPPORTED[ast.TryStar] = "TryStar"

_BIN = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul, ast.Div: operator.truediv,
        ast.FloorDiv: operator.floordiv, ast.Mod: operator.mod, ast.Pow: operator.pow}
_CMP = {ast.Eq: operator.eq, ast.NotEq: operator.ne, ast.Lt: operator.lt, ast.LtE: operator.le,
        ast.Gt: operator.gt, ast.GtE: operator.ge, ast.In: lambda a, b: a in b,
        ast.NotIn: lambda a, b: a not in b, ast.Is: operator.is_, ast.IsNot: operator.is_not}

_STR_METHODS = {"upper", "lower", "strip", "lstrip", "rstrip", "split", "join", "replace", "find", "count",
                "startswith", "endswith", "isdigit", "isalpha", "title", "capitalize", "index"}
_LIST_METHODS = {"append", "pop", "insert", "index", "count", "extend", "remove"}
_MAX_INT_BITS = 4096  # results larger than this are refused (bounded work per step)


def _check_size(v):
    if isinstance(v, int) and not isinstance(v, bool) and v.bit_length() > _MAX_INT_BITS:
        raise _Fail("OverflowError", "integer too large")
    if isinstance(v, (str, list, tuple)) and len(v) > 1_000_000:
        raise _Fail("MemoryError", "sequence too large")
    return v


def _repr(v) -> str:
    if isinstance(v, str):
        return repr(v)
    return _str(v)


def _str(v) -> str:
    if isinstance(v, list):
        return "[" + ", ".join(_repr(x) for x in v) + "]"
    if isinstance(v, tuple):
        inner = ", ".join(_repr(x) for x in v)
        return "(" + inner + ("," if len(v) == 1 else "") + ")"
    if isinstance(v, _UserFn):
        return f"<function {v.name}>"
    return str(v)


class _Machine:
    def __init__(self, max_steps: int, max_output: int, max_depth: int):
        self.max_steps, self.max_output, self.max_depth = max_steps, max_output, max_depth
        self.steps = 0
        self.out: list[str] = []
        self.out_len = 0
        self.depth = 0
        self.builtins = {
            "print": self._print, "len": self._len, "range": self._range, "int": self._int, "str": _str,
            "float": self._float, "bool": bool, "abs": abs, "min": self._minmax(min), "max": self._minmax(max),
            "sum": self._sum, "sorted": self._sorted, "reversed": lambda x: list(reversed(self._seq(x))),
            "enumerate": lambda x, start=0: [(i + start, v) for i, v in enumerate(self._seq(x))],
            "zip": lambda *xs: [tuple(t) for t in zip(*[self._seq(x) for x in xs])],
            "list": lambda x=(): list(self._seq(x)), "round": round, "divmod": self._divmod,
        }

    # -------------------------------------------------------------------- limits / output
    def tick(self):
        self.steps += 1
        if self.steps > self.max_steps:
            raise _Stop("StepLimit: exceeded max_steps")

    def emit(self, text: str):
        room = self.max_output - self.out_len
        if len(text) > room:
            self.out.append(text[:max(room, 0)])
            self.out_len = self.max_output
            raise _Stop("OutputLimit: exceeded max_output")
        self.out.append(text)
        self.out_len += len(text)

    # ------------------------------------------------------------------------ builtins
    def _print(self, *args, sep=" ", end="\n"):
        if not isinstance(sep, str) or not isinstance(end, str):
            raise _Fail("TypeError", "sep and end must be strings")
        self.emit(sep.join(_str(a) for a in args) + end)

    def _seq(self, x):
        if isinstance(x, (list, tuple, str, range)):
            return x
        raise _Fail("TypeError", f"'{type(x).__name__}' object is not iterable")

    def _len(self, x):
        return len(self._seq(x))

    def _range(self, *a):
        if not all(isinstance(x, int) for x in a) or not 1 <= len(a) <= 3:
            raise _Fail("TypeError", "range() takes 1 to 3 integer arguments")
        if len(a) == 3 and a[2] == 0:
            raise _Fail("ValueError", "range() arg 3 must not be zero")
        r = range(*a)
        if len(r) > self.max_steps:  # cannot be iterated within the budget anyway
            raise _Stop("StepLimit: exceeded max_steps")
        return r

    def _int(self, x=0, *base):
        try:
            return int(x, *base)
        except (ValueError, TypeError) as e:
            raise _Fail(type(e).__name__, str(e)) from None

    def _float(self, x=0.0):
        try:
            return float(x)
        except (ValueError, TypeError) as e:
            raise _Fail(type(e).__name__, str(e)) from None

    def _minmax(self, fn):
        def f(*a):
            seq = list(self._seq(a[0])) if len(a) == 1 else list(a)
            if not seq:
                raise _Fail("ValueError", f"{fn.__name__}() arg is an empty sequence")
            try:
                return fn(seq)
            except TypeError as e:
                raise _Fail("TypeError", str(e)) from None
        return f

    def _sum(self, x, start=0):
        try:
            return _check_size(sum(self._seq(x), start))
        except TypeError as e:
            raise _Fail("TypeError", str(e)) from None

    def _sorted(self, x, reverse=False):
        try:
            return sorted(self._seq(x), reverse=reverse)
        except TypeError as e:
            raise _Fail("TypeError", str(e)) from None

    def _divmod(self, a, b):
        if b == 0:
            raise _Fail("ZeroDivisionError", "integer division or modulo by zero")
        return divmod(a, b)

    # ---------------------------------------------------------------------- statements
    def block(self, body, env):
        for st in body:
            self.stmt(st, env)

    def stmt(self, n, env):
        self.tick()
        kind = type(n)
        if kind in _UNSUPPORTED:
            raise _Fail("UnsupportedSyntax", _UNSUPPORTED[kind])
        if kind is ast.Expr:
            self.expr(n.value, env)
        elif kind is ast.Assign:
            v = self.expr(n.value, env)
            for t in n.targets:
                self.assign(t, v, env)
        elif kind is ast.AugAssign:
            cur = self.expr(_as_load(n.target), env)
            self.assign(n.target, self.binop(n.op, cur, self.expr(n.value, env)), env)
        elif kind is ast.If:
            self.block(n.body if self.truth(self.expr(n.test, env)) else n.orelse, env)
        elif kind is ast.While:
            broke = False
            while self.truth(self.expr(n.test, env)):
                self.tick()
                try:
                    self.block(n.body, env)
                except _Break:
                    broke = True
                    break
                except _Continue:
                    continue
            if not broke:
                self.block(n.orelse, env)
        elif kind is ast.For:
            broke = False
            for item in list(self._seq(self.expr(n.iter, env))):
                self.tick()
                self.assign(n.target, item, env)
                try:
                    self.block(n.body, env)
                except _Break:
                    broke = True
                    break
                except _Continue:
                    continue
            if not broke:
                self.block(n.orelse, env)
        elif kind is ast.Break:
            raise _Break()
        elif kind is ast.Continue:
            raise _Continue()
        elif kind is ast.Pass:
            pass
        elif kind is ast.FunctionDef:
            if n.decorator_list:
                raise _Fail("UnsupportedSyntax", "decorators")
            a = n.args
            if a.vararg or a.kwarg or a.kwonlyargs or a.posonlyargs:
                raise _Fail("UnsupportedSyntax", "variadic or keyword-only parameters")
            env[n.name] = _UserFn(n, [self.expr(d, env) for d in a.defaults], env.globals)
        elif kind is ast.Return:
            raise _Return(None if n.value is None else self.expr(n.value, env))
        else:
            raise _Fail("UnsupportedSyntax", kind.__name__)

    def assign(self, t, v, env):
        kind = type(t)
        if kind is ast.Name:
            env[t.id] = v
        elif kind in (ast.Tuple, ast.List):
            vals = list(self._seq(v))
            if len(vals) != len(t.elts):
                raise _Fail("ValueError", f"expected {len(t.elts)} values to unpack, got {len(vals)}")
            for sub, x in zip(t.elts, vals):
                self.assign(sub, x, env)
        elif kind is ast.Subscript:
            obj = self.expr(t.value, env)
            if not isinstance(obj, list):
                raise _Fail("TypeError", f"'{type(obj).__name__}' object does not support item assignment")
            key = self.index(t.slice, env)
            try:
                obj[key] = v
            except (IndexError, TypeError) as e:
                raise _Fail(type(e).__name__, str(e)) from None
        elif kind in _UNSUPPORTED:
            raise _Fail("UnsupportedSyntax", _UNSUPPORTED[kind])
        else:
            raise _Fail("UnsupportedSyntax", f"assignment to {kind.__name__}")

    # --------------------------------------------------------------------- expressions
    def truth(self, v) -> bool:
        return bool(v)

    def expr(self, n, env):
        self.tick()
        kind = type(n)
        if kind in _UNSUPPORTED:
            raise _Fail("UnsupportedSyntax", _UNSUPPORTED[kind])
        if kind is ast.Constant:
            if isinstance(n.value, (int, float, str, bool)) or n.value is None:
                return n.value
            raise _Fail("UnsupportedSyntax", f"constant of type {type(n.value).__name__}")
        if kind is ast.Name:
            return env.lookup(n.id, self.builtins)
        if kind is ast.List:
            return [self.expr(e, env) for e in n.elts]
        if kind is ast.Tuple:
            return tuple(self.expr(e, env) for e in n.elts)
        if kind is ast.UnaryOp:
            v = self.expr(n.operand, env)
            if isinstance(n.op, ast.Not):
                return not v
            try:
                return -v if isinstance(n.op, ast.USub) else +v if isinstance(n.op, ast.UAdd) else ~v
            except TypeError as e:
                raise _Fail("TypeError", str(e)) from None
        if kind is ast.BinOp:
            return self.binop(n.op, self.expr(n.left, env), self.expr(n.right, env))
        if kind is ast.BoolOp:
            v = None
            for e in n.values:
                v = self.expr(e, env)
                if isinstance(n.op, ast.And) and not v:
                    return v
                if isinstance(n.op, ast.Or) and v:
                    return v
            return v
        if kind is ast.Compare:
            left = self.expr(n.left, env)
            for op, c in zip(n.ops, n.comparators):
                right = self.expr(c, env)
                try:
                    ok = _CMP[type(op)](left, right)
                except TypeError as e:
                    raise _Fail("TypeError", str(e)) from None
                if not ok:
                    return False
                left = right
            return True
        if kind is ast.IfExp:
            return self.expr(n.body if self.truth(self.expr(n.test, env)) else n.orelse, env)
        if kind is ast.Subscript:
            obj = self.expr(n.value, env)
            key = self.index(n.slice, env)
            if not isinstance(obj, (list, tuple, str)):
                raise _Fail("TypeError", f"'{type(obj).__name__}' object is not subscriptable")
            try:
                return obj[key]
            except IndexError as e:
                raise _Fail("IndexError", str(e)) from None
            except TypeError as e:
                raise _Fail("TypeError", str(e)) from None
        if kind is ast.ListComp:
            return self.listcomp(n, env)
        if kind is ast.JoinedStr:
            return "".join(self.fpart(p, env) for p in n.values)
        if kind is ast.Call:
            return self.call(n, env)
        if kind is ast.Attribute:
            raise _Fail("AttributeError", f"attribute access '{n.attr}' is not allowed")
        raise _Fail("UnsupportedSyntax", kind.__name__)

    def index(self, s, env):
        if isinstance(s, ast.Slice):
            parts = [None if p is None else self.expr(p, env) for p in (s.lower, s.upper, s.step)]
            if parts[2] == 0:
                raise _Fail("ValueError", "slice step cannot be zero")
            return slice(*parts)
        return self.expr(s, env)

    def binop(self, op, a, b):
        fn = _BIN.get(type(op))
        if fn is None:
            raise _Fail("UnsupportedSyntax", type(op).__name__)
        if isinstance(op, ast.Pow) and isinstance(b, int) and isinstance(a, int) and abs(b) > 4096:
            raise _Fail("OverflowError", "exponent too large")
        if isinstance(op, ast.Mult) and isinstance(a, (str, list, tuple)) and isinstance(b, int) and len(a) * b > 10**6:
            raise _Fail("MemoryError", "sequence too large")
        try:
            return _check_size(fn(a, b))
        except ZeroDivisionError as e:
            raise _Fail("ZeroDivisionError", str(e)) from None
        except (TypeError, ValueError, OverflowError) as e:
            raise _Fail(type(e).__name__, str(e)) from None

    def listcomp(self, n, env):
        inner = _Env(dict(), env)  # the loop variables live in their own scope
        out = []

        def gen(i):
            if i == len(n.generators):
                out.append(self.expr(n.elt, inner))
                return
            g = n.generators[i]
            if g.is_async:
                raise _Fail("UnsupportedSyntax", "async comprehension")
            for item in list(self._seq(self.expr(g.iter, inner))):
                self.tick()
                self.assign(g.target, item, inner)
                if all(self.truth(self.expr(c, inner)) for c in g.ifs):
                    gen(i + 1)

        gen(0)
        return out

    def fpart(self, p, env) -> str:
        if isinstance(p, ast.Constant):
            return str(p.value)
        v = self.expr(p.value, env)
        if p.conversion == ord("r"):
            v = _repr(v)
        elif p.conversion == ord("s"):
            v = _str(v)
        spec = "" if p.format_spec is None else self.expr(p.format_spec, env)
        try:
            return format(v, spec) if spec else _str(v)
        except (ValueError, TypeError) as e:
            raise _Fail(type(e).__name__, str(e)) from None

    def call(self, n, env):
        if any(isinstance(a, ast.Starred) for a in n.args) or any(k.arg is None for k in n.keywords):
            raise _Fail("UnsupportedSyntax", "starred arguments")
        if isinstance(n.func, ast.Attribute):
            return self.method(n, env)
        fn = self.expr(n.func, env)
        args = [self.expr(a, env) for a in n.args]
        kwargs = {k.arg: self.expr(k.value, env) for k in n.keywords}
        if isinstance(fn, _UserFn):
            return self.call_user(fn, args, kwargs)
        if callable(fn) and not isinstance(fn, type):
            try:
                return fn(*args, **kwargs)
            except (_Fail, _Stop):
                raise
            except TypeError as e:
                raise _Fail("TypeError", str(e)) from None
        if fn is bool:
            return bool(*args)
        raise _Fail("TypeError", f"'{type(fn).__name__}' object is not callable")

    def call_user(self, fn: _UserFn, args, kwargs):
        node = fn.node
        names = [a.arg for a in node.args.args]
        if len(args) > len(names):
            raise _Fail("TypeError", f"{fn.name}() takes {len(names)} positional arguments but {len(args)} were given")
        local = dict(zip(names, args))
        for k, v in kwargs.items():
            if k not in names:
                raise _Fail("TypeError", f"{fn.name}() got an unexpected keyword argument '{k}'")
            if k in local:
                raise _Fail("TypeError", f"{fn.name}() got multiple values for argument '{k}'")
            local[k] = v
        first_default = len(names) - len(fn.defaults)
        for i, name in enumerate(names):
            if name not in local:
                if i >= first_default:
                    local[name] = fn.defaults[i - first_default]
                else:
                    raise _Fail("TypeError", f"{fn.name}() missing required argument '{name}'")
        self.depth += 1
        if self.depth > self.max_depth:
            raise _Fail("RecursionError", "maximum recursion depth exceeded")
        try:
            self.block(node.body, _Env(local, fn.globals))
        except _Return as r:
            return r.value
        except (_Break, _Continue):
            raise _Fail("SyntaxError", "'break' or 'continue' outside loop")
        finally:
            self.depth -= 1
        return None

    def method(self, n, env):
        name = n.func.attr
        if name.startswith("_"):
            raise _Fail("AttributeError", f"attribute '{name}' is not allowed")
        obj = self.expr(n.func.value, env)
        allowed = _STR_METHODS if isinstance(obj, str) else _LIST_METHODS if isinstance(obj, list) else set()
        if name not in allowed:
            raise _Fail("AttributeError", f"'{type(obj).__name__}' object has no allowed method '{name}'")
        args = [self.expr(a, env) for a in n.args]
        kwargs = {k.arg: self.expr(k.value, env) for k in n.keywords}
        try:
            return _check_size(getattr(obj, name)(*args, **kwargs))
        except (ValueError, IndexError, TypeError) as e:
            raise _Fail(type(e).__name__, str(e)) from None


class _Env(dict):
    """A scope: its own names, then the globals (a function body sees its locals, then the
    module's names; module level uses the module dict for both)."""

    def __init__(self, local: dict, globals_: "_Env | None" = None):
        super().__init__(local)
        self.globals = self if globals_ is None else globals_

    def lookup(self, name: str, builtins: dict):
        if name in self:
            return self[name]
        if self.globals is not self and name in self.globals:
            return self.globals.lookup(name, builtins)
        if name in builtins:
            return builtins[name]
        raise _Fail("NameError", f"name '{name}' is not defined")


def _as_load(t):
    """The load form of an augmented-assignment target."""
    if isinstance(t, ast.Name):
        return ast.Name(id=t.id, ctx=ast.Load())
    if isinstance(t, ast.Subscript):
        return ast.Subscript(value=t.value, slice=t.slice, ctx=ast.Load())
    raise _Fail("UnsupportedSyntax", f"augmented assignment to {type(t).__name__}")


def run(source: str, max_steps: int = 100_000, max_output: int = 10_000, max_depth: int = 200) -> ExecResult:
    """Execute ``source``; never raises. The host recursion limit is raised for the call so that
    ``max_depth`` nested program calls (a few host frames each) fit under it."""
    import sys

    old_limit = sys.getrecursionlimit()
    sys.setrecursionlimit(max(old_limit, 40 * max_depth + 1000))
    try:
        return _run(source, max_steps, max_output, max_depth)
    finally:
        sys.setrecursionlimit(old_limit)


def _run(source: str, max_steps: int, max_output: int, max_depth: int) -> ExecResult:
    m = _Machine(max_steps, max_output, max_depth)
    try:
        tree = ast.parse(source, mode="exec")
    except SyntaxError as e:
        return ExecResult("", False, f"SyntaxError: {e.msg}", 0)
    except (ValueError, RecursionError) as e:
        return ExecResult("", False, f"SyntaxError: {e}", 0)
    error = None
    try:
        m.block(tree.body, _Env({}))
    except _Fail as e:
        error = e.text
    except _Stop as e:
        error = e.text
    except _Return:
        error = "SyntaxError: 'return' outside function"
    except (_Break, _Continue):
        error = "SyntaxError: 'break' or 'continue' outside loop"
    except RecursionError:
        error = "RecursionError: maximum recursion depth exceeded"
    return ExecResult("".join(m.out), error is None, error, m.steps)
