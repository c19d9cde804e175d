"""A small step executor with the interface of marin's (``ExecutorStep``, ``versioned``,
``output_path_of``, ``this_output_path``, ``executor_main``), as used by the reference launchers
(tiny-stories/launch.py:141-260, megagpt-speedrun/launch.py:128-573).

* A step is ``ExecutorStep(name, fn, config)``; ``fn(config)`` runs with every placeholder in the
  config resolved.
* ``versioned(v)`` marks a config value as part of the step's version. The version hashes the step
  name, every versioned value (with its position in the config) and the versions of the steps it
  depends on, so changing a versioned value -- or any upstream one -- gives a new output directory
  ``<prefix>/<name>-<hash6>``. Unversioned values (run ids, trackers) do not.
* ``output_path_of(step, sub)`` is a dependency on ``step`` resolved to its output path (joined with
  ``sub``); ``this_output_path(sub)`` resolves to the step's own output path.
* Every output directory holds ``.executor_info`` (name, version, resolved config, dependencies) and
  ``.executor_status`` (one JSON line per transition: RUNNING / SUCCESS / FAILED). SUCCESS steps are
  skipped; FAILED ones rerun only with ``--force_run_failed``. ``--dry_run`` prints the plan.
"""

from __future__ import annotations

import argparse
import dataclasses
import datetime
import hashlib
import json
import os
import sys
import traceback
from collections.abc import Callable
from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True)
class VersionedValue:
    value: Any


def versioned(value: Any) -> VersionedValue:
    return VersionedValue(value)


@dataclass(frozen=True)
class OutputPathOf:
    step: "ExecutorStep"
    name: str | None = None


def output_path_of(step: "ExecutorStep", name: str | None = None) -> OutputPathOf:
    return OutputPathOf(step, name)


@dataclass(frozen=True)
class ThisOutputPath:
    name: str | None = None


def this_output_path(name: str | None = None) -> ThisOutputPath:
    return ThisOutputPath(name)


@dataclass(frozen=True, eq=False)
class ExecutorStep:
    name: str
    fn: Callable[[Any], Any]
    config: Any
    description: str | None = None
    override_output_path: str | None = None

    def cd(self, name: str) -> OutputPathOf:
        return OutputPathOf(self, name)


# ------------------------------------------------------------------------------- traversal
def _children(obj):
    if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        return [(f.name, getattr(obj, f.name)) for f in dataclasses.fields(obj)]
    if isinstance(obj, dict):
        return list(obj.items())
    if isinstance(obj, (list, tuple)):
        return list(enumerate(obj))
    return []


def _walk(obj, path=()):
    yield path, obj
    if isinstance(obj, (VersionedValue, OutputPathOf, ThisOutputPath, ExecutorStep)):
        if isinstance(obj, VersionedValue):
            yield from _walk(obj.value, path + ("<v>",))
        return
    for k, v in _children(obj):
        yield from _walk(v, path + (k,))


def _map(obj, fn):
    """Rebuild ``obj`` with ``fn`` applied to every placeholder (bottom-up)."""
    r = fn(obj)
    if r is not obj:
        return r
    if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        changes = {f.name: _map(getattr(obj, f.name), fn) for f in dataclasses.fields(obj) if f.init}
        return dataclasses.replace(obj, **changes)
    if isinstance(obj, dict):
        return {k: _map(v, fn) for k, v in obj.items()}
    if isinstance(obj, tuple):
        return tuple(_map(v, fn) for v in obj)
    if isinstance(obj, list):
        return [_map(v, fn) for v in obj]
    return obj


def _jsonable(v):
    if dataclasses.is_dataclass(v) and not isinstance(v, type):
        return {"__type__": type(v).__name__, **{f.name: _jsonable(getattr(v, f.name)) for f in dataclasses.fields(v)}}
    if isinstance(v, dict):
        return {str(k): _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    if isinstance(v, (str, int, float, bool)) or v is None:
        return v
    if isinstance(v, VersionedValue):
        return _jsonable(v.value)
    if isinstance(v, OutputPathOf):
        return {"__output_path_of__": v.step.name, "name": v.name}
    if isinstance(v, ThisOutputPath):
        return {"__this_output_path__": v.name}
    if callable(v):
        return getattr(v, "__qualname__", repr(v))
    return repr(v)


def dependencies(step: ExecutorStep) -> list[ExecutorStep]:
    deps = []
    for _, v in _walk(step.config):
        if isinstance(v, OutputPathOf) and v.step not in deps:
            deps.append(v.step)
    return deps


# -------------------------------------------------------------------------------- executor
class Executor:
    def __init__(self, prefix: str, *, dry_run: bool = False, force_run_failed: bool = False,
                 run_only: list[str] | None = None, log=print):
        self.prefix = prefix
        self.dry_run = dry_run
        self.force_run_failed = force_run_failed
        self.run_only = run_only
        self.log = log
        self._versions: dict[int, dict] = {}
        self._paths: dict[int, str] = {}

    def version(self, step: ExecutorStep) -> dict:
        key = id(step)
        if key not in self._versions:
            vals = {"/".join(map(str, p)): _jsonable(v.value) for p, v in _walk(step.config)
                    if isinstance(v, VersionedValue)}
            self._versions[key] = {"name": step.name, "config": vals,
                                   "dependencies": [self.version(d) for d in dependencies(step)]}
        return self._versions[key]

    def output_path(self, step: ExecutorStep) -> str:
        key = id(step)
        if key not in self._paths:
            if step.override_output_path:
                p = step.override_output_path
            else:
                h = hashlib.md5(json.dumps(self.version(step), sort_keys=True).encode()).hexdigest()[:6]
                p = os.path.join(self.prefix, f"{step.name}-{h}")
            self._paths[key] = p
        return self._paths[key]

    def instantiate(self, step: ExecutorStep):
        own = self.output_path(step)

        def fn(v):
            if isinstance(v, VersionedValue):
                return _map(v.value, fn)
            if isinstance(v, OutputPathOf):
                base = self.output_path(v.step)
                return base if v.name is None else os.path.join(base, v.name)
            if isinstance(v, ThisOutputPath):
                return own if v.name is None else os.path.join(own, v.name)
            return v

        return _map(step.config, fn)

    @staticmethod
    def status(path: str) -> str | None:
        sp = os.path.join(path, ".executor_status")
        if not os.path.exists(sp):
            return None
        last = None
        with open(sp) as f:
            for line in f:
                if line.strip():
                    last = json.loads(line)["status"]
        return last

    @staticmethod
    def _append_status(path: str, status: str) -> None:
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, ".executor_status"), "a") as f:
            f.write(json.dumps({"date": datetime.datetime.now().isoformat(), "status": status}) + "\n")

    def plan(self, steps: list[ExecutorStep]) -> list[ExecutorStep]:
        order: list[ExecutorStep] = []
        seen: set[int] = set()
        visiting: set[int] = set()

        def visit(s):
            if id(s) in seen:
                return
            if id(s) in visiting:
                raise ValueError(f"dependency cycle at step {s.name}")
            visiting.add(id(s))
            for d in dependencies(s):
                visit(d)
            visiting.discard(id(s))
            seen.add(id(s))
            order.append(s)

        for s in steps:
            visit(s)
        if self.run_only:
            keep = set()
            for s in order:
                if any(s.name == r or s.name.startswith(r.rstrip("*")) for r in self.run_only):
                    keep.add(id(s))
                    stack = list(dependencies(s))
                    while stack:
                        d = stack.pop()
                        keep.add(id(d))
                        stack += dependencies(d)
            order = [s for s in order if id(s) in keep]
        return order

    def run(self, steps: list[ExecutorStep]) -> dict[str, str]:
        results = {}
        for step in self.plan(steps):
            path = self.output_path(step)
            st = self.status(path)
            results[step.name] = path
            if self.dry_run:
                self.log(f"[dry-run] {step.name} -> {path} (status: {st or 'not run'})")
                continue
            if st == "SUCCESS":
                self.log(f"[executor] skip {step.name}: already succeeded at {path}")
                continue
            if st == "FAILED" and not self.force_run_failed:
                raise RuntimeError(f"step {step.name} failed before at {path}; pass --force_run_failed to retry")
            cfg = self.instantiate(step)
            os.makedirs(path, exist_ok=True)
            with open(os.path.join(path, ".executor_info"), "w") as f:
                json.dump({"name": step.name, "description": step.description, "version": self.version(step),
                           "config": _jsonable(cfg), "output_path": path,
                           "dependencies": [self.output_path(d) for d in dependencies(step)]}, f, indent=1)
            self._append_status(path, "RUNNING")
            self.log(f"[executor] run {step.name} -> {path}")
            try:
                step.fn(cfg)
            except BaseException:
                self._append_status(path, "FAILED")
                traceback.print_exc()
                raise
            self._append_status(path, "SUCCESS")
        return results


def executor_main(steps: list[ExecutorStep], description: str | None = None, argv: list[str] | None = None,
                  default_prefix: str | None = None) -> dict[str, str]:
    ap = argparse.ArgumentParser(description=description)
    ap.add_argument("--prefix", default=os.environ.get("MARIN_PREFIX", default_prefix or "outputs"))
    ap.add_argument("--dry_run", action="store_true")
    ap.add_argument("--force_run_failed", action="store_true")
    ap.add_argument("--run_only", nargs="*", default=None)
    args, _ = ap.parse_known_args(sys.argv[1:] if argv is None else argv)
    ex = Executor(args.prefix, dry_run=args.dry_run, force_run_failed=args.force_run_failed, run_only=args.run_only)
    return ex.run(steps)
