"""Executor: versioned output paths, dependency resolution, skip-on-success, failure handling,
dry run and run_only."""

import json
import os
from dataclasses import dataclass

import pytest

from marin_experiments_b200.executor import (Executor, ExecutorStep, executor_main, output_path_of, this_output_path,
                                             versioned)


@dataclass(frozen=True)
class Cfg:
    out: object
    n: object = 1
    src: object = None
    note: str = ""


CALLS = []


def produce(c: Cfg):
    CALLS.append(("produce", c.n))
    os.makedirs(c.out, exist_ok=True)
    with open(os.path.join(c.out, "data.txt"), "w") as f:
        f.write(str(c.n))


def consume(c: Cfg):
    CALLS.append(("consume", c.src))
    with open(c.src) as f:
        v = int(f.read())
    with open(os.path.join(c.out, "sum.txt"), "w") as f:
        f.write(str(v + c.n))


def fail(c: Cfg):
    raise RuntimeError("boom")


def _steps(n=1, note=""):
    a = ExecutorStep("raw/a", produce, Cfg(out=this_output_path(), n=versioned(n), note=note))
    b = ExecutorStep("train/b", consume, Cfg(out=this_output_path(), n=versioned(10), src=output_path_of(a, "data.txt")))
    return a, b


def test_run_skip_and_versions(tmp_path):
    CALLS.clear()
    a, b = _steps()
    ex = Executor(str(tmp_path))
    res = ex.run([b])  # a is pulled in as a dependency
    assert [c[0] for c in CALLS] == ["produce", "consume"]
    assert open(os.path.join(res["train/b"], "sum.txt")).read() == "11"
    assert Executor.status(res["raw/a"]) == "SUCCESS"
    info = json.load(open(os.path.join(res["train/b"], ".executor_info")))
    assert info["dependencies"] == [res["raw/a"]]
    CALLS.clear()
    a2, b2 = _steps(note="unversioned change")
    res2 = Executor(str(tmp_path)).run([b2])
    assert CALLS == [] and res2 == res  # same versions -> skipped
    a3, b3 = _steps(n=2)
    res3 = Executor(str(tmp_path)).run([b3])
    assert res3["raw/a"] != res["raw/a"] and res3["train/b"] != res["train/b"]  # upstream change propagates
    assert open(os.path.join(res3["train/b"], "sum.txt")).read() == "12"


def test_failure_and_force(tmp_path):
    s = ExecutorStep("bad", fail, Cfg(out=this_output_path()))
    with pytest.raises(RuntimeError):
        Executor(str(tmp_path)).run([s])
    path = Executor(str(tmp_path)).output_path(s)
    assert Executor.status(path) == "FAILED"
    with pytest.raises(RuntimeError, match="force_run_failed"):
        Executor(str(tmp_path)).run([s])
    with pytest.raises(RuntimeError, match="boom"):
        Executor(str(tmp_path), force_run_failed=True).run([s])


def test_dry_run_and_run_only(tmp_path, capsys):
    CALLS.clear()
    a, b = _steps()
    executor_main([b], argv=["--prefix", str(tmp_path), "--dry_run"])
    assert CALLS == []
    assert "[dry-run] train/b" in capsys.readouterr().out
    Executor(str(tmp_path), run_only=["raw/a"]).run([b])
    assert CALLS == [("produce", 1)]


def test_accelerator_switch(monkeypatch):
    import pytest

    from marin_experiments_b200.train import run

    monkeypatch.setenv("ACCELERATOR", "cpu")
    assert run._device().type == "cpu"
    monkeypatch.setenv("ACCELERATOR", "tpu")
    with pytest.raises(ValueError, match="cpu or gpu"):
        run._device()
    import torch

    if not torch.cuda.is_available():
        monkeypatch.setenv("ACCELERATOR", "gpu")
        with pytest.raises(RuntimeError, match="no CUDA device"):
            run._device()
