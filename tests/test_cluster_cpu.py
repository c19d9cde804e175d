"""Job dispatch: submit / wait / retry on the local scheduler (GPU slots as plain integers, no
GPU used) and the SSH client's remote command (fake runner)."""

import json
import os
import time

import pytest

from marin_experiments_b200 import cluster as C


def _write(path, text):
    with open(path, "w") as f:
        f.write(text)


def _train_entry(cfg):
    # stands in for a training entry point: records its config and the forwarded environment
    _write(cfg["out"], json.dumps({"cfg": cfg["value"], "env": os.environ.get("MXK_TEST_FORWARDED")}))


def test_dispatch_runs_callable_with_forwarded_env(tmp_path, monkeypatch):
    monkeypatch.setenv("MXK_TEST_FORWARDED", "yes")
    monkeypatch.setenv("PYTHONPATH", os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    client = C.LocalClient(str(tmp_path / "jobs"), gpus=[])
    out = str(tmp_path / "out.json")
    job = C.dispatch_grug_training_run(run_id="my run/1", config={"out": out, "value": 7}, local_entrypoint=_train_entry,
                                       resources=C.ResourceConfig(gpus=0), client=client, max_retries_failure=0)
    assert job.status() == "SUCCEEDED" and job.job_id == "grug-train-my-run-1"
    assert json.load(open(out)) == {"cfg": 7, "env": "yes"}
    assert json.load(open(os.path.join(job.dir, "state.json")))["state"] == "SUCCEEDED"


def test_retry_then_success_and_failure(tmp_path):
    client = C.LocalClient(str(tmp_path / "jobs"), gpus=[])
    marker = tmp_path / "tried"
    flaky = C.Entrypoint.from_command("sh", "-c", f"if [ -e {marker} ]; then exit 0; else touch {marker}; exit 3; fi")
    h = client.submit(C.JobRequest("flaky", flaky, C.ResourceConfig(gpus=0), max_retries_failure=1))
    assert h.wait() == "SUCCEEDED" and h.attempts == 2
    bad = client.submit(C.JobRequest("bad", C.Entrypoint.from_command("sh", "-c", "exit 5"), C.ResourceConfig(gpus=0),
                                     max_retries_failure=2))
    with pytest.raises(C.JobFailed, match="exit code 5"):
        bad.wait()
    assert bad.attempts == 3


def test_gpu_slots_first_come_first_served(tmp_path):
    """Jobs get disjoint GPU sets; a job waits until enough GPUs are free, in submission order."""
    client = C.LocalClient(str(tmp_path / "jobs"), gpus=[0, 1, 2])
    log = tmp_path / "log"

    def job(name, gpus, sleep):
        cmd = f"echo {name} start $CUDA_VISIBLE_DEVICES $(date +%s.%N) >> {log}; sleep {sleep}; " \
              f"echo {name} end $(date +%s.%N) >> {log}"
        return client.submit(C.JobRequest(name, C.Entrypoint.from_command("sh", "-c", cmd), C.ResourceConfig(gpus=gpus)))

    a = job("a", 2, 0.6)
    b = job("b", 2, 0.1)  # must wait for a (only one GPU left)
    c = job("c", 1, 0.1)  # behind b in the queue
    for h in (a, b, c):
        h.wait(timeout=30)
    lines = [ln.split() for ln in open(log).read().splitlines()]
    ev = {(ln[0], ln[1]): ln for ln in lines}
    assert len(ev[("a", "start")][2].split(",")) == 2
    assert float(ev[("b", "start")][3]) >= float(ev[("a", "end")][2]) - 1e-3
    # c (one GPU) could have started beside a; in submission order it waits behind b, so it starts
    # only after a ends (b and c then start together, in either order inside their shells)
    assert float(ev[("c", "start")][3]) >= float(ev[("a", "end")][2]) - 1e-3
    with pytest.raises(ValueError, match="needs 4 GPUs"):
        client.submit(C.JobRequest("big", C.Entrypoint.from_command("true"), C.ResourceConfig(gpus=4)))


def test_cancel_pending_job(tmp_path):
    client = C.LocalClient(str(tmp_path / "jobs"), gpus=[0])
    long = client.submit(C.JobRequest("long", C.Entrypoint.from_command("sleep", "30"), C.ResourceConfig(gpus=1)))
    queued = client.submit(C.JobRequest("queued", C.Entrypoint.from_command("true"), C.ResourceConfig(gpus=1)))
    time.sleep(0.3)
    queued.cancel()
    long.cancel()
    assert long.wait(raise_on_failure=False, timeout=10) == "KILLED"
    assert queued.wait(raise_on_failure=False, timeout=10) == "KILLED"


class _FakeRunner:
    def __init__(self, codes):
        self.codes, self.cmds, self.puts = list(codes), [], []

    def run(self, command, timeout=None):
        self.cmds.append(command)
        return self.codes.pop(0) if self.codes else 0

    def put(self, local, remote):
        self.puts.append((local, remote))


def test_ssh_client_command_and_retry(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    r = _FakeRunner([1, 0])
    client = C.SSHClient(r, workdir="/srv/repo")
    h = client.submit(C.JobRequest("sweep arm", C.Entrypoint.from_command("python", "-m", "x.y", "--a", "b c"),
                                   env_vars={"SP_EP": "8", "NCCL_DEBUG": "INFO"}, max_retries_failure=1))
    assert h.wait(timeout=10) == "SUCCEEDED" and h.attempts == 2
    cmd = r.cmds[0]
    assert cmd.startswith("cd /srv/repo && mkdir -p jobs/sweep-arm && env NCCL_DEBUG=INFO SP_EP=8 python -m x.y")
    assert "'b c'" in cmd and cmd.endswith("> jobs/sweep-arm/job.log 2>&1")


def test_forwarded_env_filter():
    env = {"NCCL_ALGO": "Ring", "MXK_EP_IMPL": "peer", "CUDA_VISIBLE_DEVICES": "0", "HOME": "/root", "SP_EP": "8"}
    assert C.forwarded_env_vars(env) == {"NCCL_ALGO": "Ring", "MXK_EP_IMPL": "peer", "SP_EP": "8"}
