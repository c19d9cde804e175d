"""Named sweeps: plan expansion and local job execution."""

import sys

import pytest

from marin_experiments_b200.experiments import megagpt, sweeps
from marin_experiments_b200.utils import analysis


def test_plan_expands_arms():
    jobs = sweeps.plan("anchor", gpus=8, tag="t1")
    assert [j.name for j in jobs] == ["t1-e64k4", "t1-e64k8", "t1-e128k8", "t1-e256k8"]
    j = jobs[2]
    assert j.env["SP_EXPERTS"] == "128" and j.env["SP_TOPK"] == "8" and j.env["SP_EP"] == "8"
    assert j.env["SP_TAG"] == "t1-e128k8" and j.env["SP_HIDDEN"] == sweeps.BASE["SP_HIDDEN"]
    assert "torch.distributed.run" in j.argv and "--nproc-per-node=8" in j.argv and "127.0.0.1" in j.argv
    assert j.argv[-2:] == ["-m", sweeps.LAUNCHER]
    # per-arm GPU counts and batch per GPU (weak scaling)
    sc = {j.name: j for j in sweeps.plan("weak", tag="s")}
    assert sc["s-g1"].gpus == 1 and sc["s-g1"].argv == [sys.executable, "-m", sweeps.LAUNCHER]
    assert sc["s-g4"].env["SP_BATCH"] == "128" and sc["s-g4"].env["SP_EP"] == "4"
    assert [j.name for j in sweeps.plan("lever", only=["embed512"], tag="x")] == ["x-embed512"]
    with pytest.raises(KeyError):
        sweeps.plan("lever", only=["nope"])
    assert sweeps.plan("dp", gpus=2)[1].env["SP_EP"] == "1"


def test_arms_are_launchable():
    """Every arm's environment builds a launch config (and the salted run id differs per tag)."""
    for name in sweeps.SWEEPS:
        if name == "pp":
            continue
        for job in sweeps.plan(name, gpus=8, tag="c"):
            env = {k: v for k, v in job.env.items() if k != "SP_PP_MODE"}
            launch, arm = megagpt.make_launch(env)
            assert arm.startswith("[arm] ")
            assert "SP_TAG" in job.env


def test_run_jobs_and_table(tmp_path, capsys):
    fake = {"demo": {"fast": {"X_TOK": "900000"}, "slow": {"X_TOK": "100000"},
                     "oom": {"X_TOK": "0", "X_FAIL": "1"}}}
    code = ("import os\n"
            "if os.environ.get('X_FAIL'):\n"
            "    raise SystemExit('torch.OutOfMemoryError: CUDA out of memory')\n"
            "print('[arm] ' + os.environ['SP_TAG'] + '  mode=fixed D=1536 d_e=1536(factorized=False) seq=2048 E=64 "
            "k=4 min_k=0 coef=0.0 nominal_active_frac=6.25% batch=32 steps=12 budget=1e18')\n"
            "for s in range(12):\n"
            "    print(f\"[THRUPUT] step={s} dt=0.500s tok_s={int(os.environ['X_TOK']) + s} mfu=0.2000 bs=32\")\n")
    jobs = sweeps.plan("demo", gpus=1, tag="d", sweeps=fake)
    for j in jobs:
        j.argv = [sys.executable, "-c", code]
    logs = sweeps.run(jobs, str(tmp_path), timeout_s=60)
    runs = analysis.analyze_logs(logs, warmup=8)
    assert runs[0].tok_s == 900009.5 and runs[1].tok_s == 100009.5 and runs[2].failure == "oom"
    table = analysis.sweep_table(runs).splitlines()
    assert "d-fast" in table[2] and "d-slow" in table[3] and "oom" in table[4]
    sweeps.run(jobs[:1], str(tmp_path / "dry"), dry_run=True)
    assert "[d-fast] gpus=1" in capsys.readouterr().out


def test_run_timeout_kills_only_the_job(tmp_path):
    jobs = sweeps.plan("demo", gpus=1, tag="to", sweeps={"demo": {"hang": {}}})
    jobs[0].argv = [sys.executable, "-c", "import time; print('start', flush=True); time.sleep(60)"]
    logs = sweeps.run(jobs, str(tmp_path), timeout_s=2)
    text = open(logs[0]).read()
    assert "killed after 2s" in text and "exit timeout" in text


def test_diag_side_entries_dispatch(monkeypatch):
    from marin_experiments_b200.benchmarks import diag

    called = []
    monkeypatch.setitem(diag.MODES, "fit", lambda: called.append("fit"))
    monkeypatch.setenv("SP_DIAG", "fit")
    assert megagpt.main([]) is None and called == ["fit"]
    with pytest.raises(SystemExit):
        diag.main("bogus")
    assert set(diag.MODES) == {"ragged", "ring", "fit", "attn"}


def test_submit_arms_to_scheduler(tmp_path):
    """Arms sent to the node scheduler run side by side on its GPUs; their logs feed the same table."""
    from marin_experiments_b200 import cluster as C

    code = ("import os, time\n"
            "print('[arm] ' + os.environ['SP_TAG'] + '  mode=fixed D=1536 d_e=1536(factorized=False) seq=2048 E=64 "
            "k=4 min_k=0 coef=0.0 nominal_active_frac=6.25% batch=32 steps=12 budget=1e18')\n"
            "for s in range(12):\n"
            "    print(f\"[THRUPUT] step={s} dt=0.500s tok_s={int(os.environ['X_TOK']) + s} mfu=0.2000 bs=32\")\n"
            "print('devices', os.environ['CUDA_VISIBLE_DEVICES'])\n")
    fake = {"demo": {"a": {"X_TOK": "500000"}, "b": {"X_TOK": "700000"}}}
    jobs = sweeps.plan("demo", gpus=1, tag="q", sweeps=fake)
    for j in jobs:
        j.argv = [sys.executable, "-c", code]
    client = C.LocalClient(str(tmp_path / "jobs"), gpus=[0, 1])
    handles = sweeps.submit(jobs, client, timeout_s=120)
    logs = sweeps.collect(handles, [j.name for j in jobs], str(tmp_path / "logs"))
    runs = analysis.analyze_logs(logs, warmup=8)
    assert runs[0].tok_s == 500009.5 and runs[1].tok_s == 700009.5
    devs = {open(p).read().split("devices ")[1].split()[0] for p in logs}
    assert devs <= {"0", "1"} and "SUCCEEDED" in open(logs[0]).read()
    # a torchrun arm is handed to the client as the plain module (the client adds torchrun itself)
    two = sweeps.plan("anchor", gpus=2, tag="t", only=["e64k4"])[0]

    class Rec:
        def submit(self, req):
            self.req = req
            return req

    r = Rec()
    sweeps.submit([two], r)
    assert list(r.req.entrypoint.command) == [sys.executable, "-m", sweeps.LAUNCHER] and r.req.resources.gpus == 2


def test_reference_grids_and_init_from(monkeypatch, capsys):
    for name in ("lossab", "best", "scale", "scale2", "scale3", "run2", "cool", "eval", "weak"):
        assert name in sweeps.SWEEPS
    la = {j.name: j for j in sweeps.plan("lossab", gpus=8, tag="l")}
    assert la["l-b_bigE"].env["SP_EXPERTS"] == "256" and la["l-a_thin"].env["SP_DATA"] == "datakit"
    launch, _ = megagpt.make_launch(la["l-a_thin"].env)
    assert launch.data.source == "remote" and launch.data.mix == "nemotron"
    cool = sweeps.plan("cool", gpus=8, tag="c")[0]
    assert megagpt.make_launch(cool.env)[0].data.mix == "sft-chat"
    with pytest.raises(SystemExit, match="needs --init-from"):
        sweeps.main(["cool", "--dry-run"])
    assert sweeps.main(["eval", "--dry-run", "--init-from", "/ckpt/run2", "--log-dir", "/tmp/x"]) == 0
    assert "SP_INIT_FROM=/ckpt/run2" in capsys.readouterr().out
