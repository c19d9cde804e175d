"""Job dispatch: submit a training entry point (or command) as a job and wait for it.

The reference hands its train entry points to a cluster client (megagpt-speedrun/dispatch.py:49-69:
a ``JobRequest`` of name, entry point, resources, environment and failure-retry count goes to
``current_client().submit`` and the dispatcher blocks in ``job.wait(raise_on_failure=True)``;
megagpt-speedrun/iris_jobs.py:302-369 submits sweep arms as commands). Its clients are cloud
schedulers; this module gives the same surface over the machines a B200 user has:

* ``LocalClient`` runs jobs on this node: each job gets whole GPUs from the node's pool
  (``CUDA_VISIBLE_DEVICES``), jobs wait in submission order until their GPUs are free, a
  multi-GPU job runs its entry point under ``torch.distributed.run`` on 127.0.0.1, every job runs in
  its own process group with its log, state and exit code under ``<root>/<job name>/``, and a
  failed job is retried up to ``max_retries_failure`` times;
* ``SSHClient`` runs the same job command on another host through a ``runner`` (paramiko by
  default: environment, working directory, log file and exit code on the remote side), one job
  per host at a time.

A callable entry point is serialised with cloudpickle next to the job and executed by
``python -m marin_experiments_b200.cluster run <file>``, so the job runs the caller's function with
its arguments (the reference's ``Entrypoint.from_callable``). ``dispatch_grug_training_run`` is the
reference's helper: sanitised job name, forwarded runtime environment, submit, wait, raise on
failure. The client comes from ``MXK_CLUSTER`` (``local`` by default, ``ssh://[user@]host[:port]``).
"""

from __future__ import annotations

import dataclasses
import json
import os
import re
import shlex
import signal
import subprocess
import sys
import threading
import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field

# Runtime environment forwarded from the dispatcher into jobs (jobs do not inherit the submitting
# shell): communication and runtime tuning of this stack and the launcher's arms.
FORWARDED_ENV_PREFIXES = ("NCCL_", "CUDA_LAUNCH_BLOCKING", "TORCH_", "MXK_", "SP_", "GRUG_", "MOE_PP_")
FORWARDED_ENV_EXCLUDE = ("CUDA_VISIBLE_DEVICES",)  # assigned per job by the scheduler


def forwarded_env_vars(environ: dict[str, str] | None = None) -> dict[str, str]:
    env = os.environ if environ is None else environ
    return {k: v for k, v in env.items() if k.startswith(FORWARDED_ENV_PREFIXES) and k not in FORWARDED_ENV_EXCLUDE}


def safe_job_suffix(run_id: str) -> str:
    """Job names allow letters, digits, ``_``, ``.`` and ``-``."""
    return re.sub(r"[^A-Za-z0-9_.-]+", "-", run_id)


@dataclass(frozen=True)
class ResourceConfig:
    gpus: int = 1
    cpu: float = 8.0
    memory: str = "64GB"


@dataclass(frozen=True)
class Entrypoint:
    """A command, or a callable with its arguments (run through cloudpickle)."""

    command: tuple[str, ...] | None = None
    fn: Callable | None = None
    args: tuple = ()
    kwargs: dict = field(default_factory=dict)

    @staticmethod
    def from_command(*argv: str) -> "Entrypoint":
        return Entrypoint(command=tuple(argv))

    @staticmethod
    def from_callable(fn: Callable, args: Sequence = (), kwargs: dict | None = None) -> "Entrypoint":
        return Entrypoint(fn=fn, args=tuple(args), kwargs=dict(kwargs or {}))


@dataclass(frozen=True)
class JobRequest:
    name: str
    entrypoint: Entrypoint
    resources: ResourceConfig = field(default_factory=ResourceConfig)
    env_vars: dict[str, str] = field(default_factory=dict)
    max_retries_failure: int = 0
    timeout_s: float | None = None


class JobFailed(RuntimeError):
    pass


# ------------------------------------------------------------------------------ job command
def _write_payload(req: JobRequest, job_dir: str) -> list[str]:
    """The job's argv; a callable is pickled into ``job_dir/entry.pkl`` first."""
    if req.entrypoint.command is not None:
        return list(req.entrypoint.command)
    import cloudpickle

    # Functions of this package and of installed libraries are pickled by reference (the job
    # imports them); a function defined in a user's script or test file travels by value.
    mod = sys.modules.get(getattr(req.entrypoint.fn, "__module__", ""), None)
    by_value = None
    if mod is not None and mod.__name__ != "__main__":
        f = getattr(mod, "__file__", "") or ""
        pkg = os.path.dirname(os.path.abspath(__file__))
        if not (f.startswith(pkg) or "site-packages" in f or f.startswith(sys.prefix)):
            by_value = mod
            cloudpickle.register_pickle_by_value(mod)
    path = os.path.join(job_dir, "entry.pkl")
    try:
        with open(path, "wb") as f:
            cloudpickle.dump((req.entrypoint.fn, req.entrypoint.args, req.entrypoint.kwargs), f)
    finally:
        if by_value is not None:
            cloudpickle.unregister_pickle_by_value(by_value)
    return [sys.executable, "-m", "marin_experiments_b200.cluster", "run", path]


def _job_argv(req: JobRequest, base: list[str], port: int) -> list[str]:
    """Multi-GPU Python jobs run one rank per GPU under torch.distributed.run on 127.0.0.1."""
    n = req.resources.gpus
    if n <= 1 or base[:1] != [sys.executable]:
        return base
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
            "--master-addr", "127.0.0.1", "--master-port", str(port)] + base[1:]


# ------------------------------------------------------------------------------ local client
class JobHandle:
    def __init__(self, client, req: JobRequest, job_dir: str):
        self.client, self.request, self.dir = client, req, job_dir
        self.job_id = os.path.basename(job_dir)
        self._done = threading.Event()
        self.state = "PENDING"
        self.exit_code: int | None = None
        self.attempts = 0

    def _set(self, state: str, code: int | None = None) -> None:
        self.state, self.exit_code = state, code
        with open(os.path.join(self.dir, "state.json"), "w") as f:
            json.dump({"state": state, "exit_code": code, "attempts": self.attempts, "time": time.time()}, f)
        if state in ("SUCCEEDED", "FAILED", "KILLED"):
            self._done.set()

    def status(self) -> str:
        return self.state

    def log_path(self) -> str:
        return os.path.join(self.dir, "job.log")

    def wait(self, *, raise_on_failure: bool = True, timeout: float | None = None) -> str:
        if not self._done.wait(timeout):
            raise TimeoutError(f"job {self.job_id} still {self.state} after {timeout} s")
        if raise_on_failure and self.state != "SUCCEEDED":
            raise JobFailed(f"job {self.job_id} {self.state} (exit code {self.exit_code}); log: {self.log_path()}")
        return self.state

    def cancel(self) -> None:
        self.client._cancel(self)


class LocalClient:
    """Jobs on this node's GPUs, first come first served."""

    def __init__(self, root: str = "jobs", gpus: Sequence[int] | None = None, base_port: int = 29700):
        self.root = root
        os.makedirs(root, exist_ok=True)
        if gpus is None:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                gpus = [int(x) for x in vis.split(",") if x.strip().isdigit()]
            else:
                try:
                    import torch

                    gpus = list(range(torch.cuda.device_count()))
                except Exception:
                    gpus = []
        self.free = list(gpus)
        self.total = len(self.free)
        self.port = base_port
        self.cv = threading.Condition()
        self.queue: list[JobHandle] = []
        self.procs: dict[str, subprocess.Popen] = {}

    def submit(self, req: JobRequest) -> JobHandle:
        need = req.resources.gpus
        if need > max(self.total, 0) and need > 0 and self.total > 0:
            raise ValueError(f"job {req.name} needs {need} GPUs; this node has {self.total}")
        job_dir = os.path.join(self.root, safe_job_suffix(req.name))
        os.makedirs(job_dir, exist_ok=True)
        h = JobHandle(self, req, job_dir)
        h._set("PENDING")
        with self.cv:
            self.queue.append(h)
        threading.Thread(target=self._run, args=(h,), daemon=True).start()
        return h

    def _take(self, h: JobHandle) -> list[int] | None:
        need = h.request.resources.gpus if self.total else 0
        with self.cv:
            while not (self.queue and self.queue[0] is h and len(self.free) >= need):
                if h.state == "KILLED":
                    return None
                self.cv.wait(0.2)
            self.queue.pop(0)
            got, self.free = self.free[:need], self.free[need:]
            self.port += 1
            self.cv.notify_all()
            return got

    def _give(self, gpus: list[int]) -> None:
        with self.cv:
            self.free = sorted(self.free + gpus)
            self.cv.notify_all()

    def _run(self, h: JobHandle) -> None:
        gpus = self._take(h)
        if gpus is None:
            return
        req = h.request
        try:
            base = _write_payload(req, h.dir)
            argv = _job_argv(req, base, self.port)
            env = dict(os.environ)
            env.update(req.env_vars)
            if self.total:
                env["CUDA_VISIBLE_DEVICES"] = ",".join(str(g) for g in gpus)
            with open(os.path.join(h.dir, "job.cmd"), "w") as f:
                f.write(" ".join(shlex.quote(a) for a in argv) + "\n")
            while True:
                h.attempts += 1
                h._set("RUNNING")
                with open(h.log_path(), "ab") as log:
                    p = subprocess.Popen(argv, env=env, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
                    self.procs[h.job_id] = p
                    try:
                        code = p.wait(timeout=req.timeout_s)
                    except subprocess.TimeoutExpired:
                        os.killpg(p.pid, signal.SIGKILL)
                        code = p.wait()
                if h.state == "KILLED":
                    return
                if code == 0:
                    h._set("SUCCEEDED", 0)
                    return
                if h.attempts > req.max_retries_failure:
                    h._set("FAILED", code)
                    return
        finally:
            self.procs.pop(h.job_id, None)
            self._give(gpus)

    def _cancel(self, h: JobHandle) -> None:
        h._set("KILLED", None)
        p = self.procs.get(h.job_id)
        if p is not None and p.poll() is None:
            os.killpg(p.pid, signal.SIGKILL)
        with self.cv:
            if h in self.queue:
                self.queue.remove(h)
            self.cv.notify_all()


# -------------------------------------------------------------------------------- SSH client
class ParamikoRunner:
    """Runs a shell command on a host over SSH and returns its exit code (paramiko)."""

    def __init__(self, host: str, user: str | None = None, port: int = 22):
        self.host, self.user, self.port = host, user, port

    def run(self, command: str, timeout: float | None = None) -> int:
        import paramiko

        c = paramiko.SSHClient()
        c.load_system_host_keys()
        c.set_missing_host_key_policy(paramiko.RejectPolicy())
        c.connect(self.host, port=self.port, username=self.user)
        try:
            _, out, _ = c.exec_command(command, timeout=timeout)
            return out.channel.recv_exit_status()
        finally:
            c.close()

    def put(self, local: str, remote: str) -> None:
        import paramiko

        c = paramiko.SSHClient()
        c.load_system_host_keys()
        c.set_missing_host_key_policy(paramiko.RejectPolicy())
        c.connect(self.host, port=self.port, username=self.user)
        try:
            sftp = c.open_sftp()
            sftp.put(local, remote)
            sftp.close()
        finally:
            c.close()


class SSHClient:
    """Jobs on another host: ``cd <workdir> && env ... <argv> > <remote job dir>/job.log``, the exit
    code returned by the runner (retried like a local job)."""

    def __init__(self, runner, *, workdir: str = ".", remote_root: str = "jobs", python: str = "python"):
        self.runner, self.workdir, self.remote_root, self.python = runner, workdir, remote_root, python
        self.local_root = os.path.join("jobs", "ssh")
        os.makedirs(self.local_root, exist_ok=True)
        self.lock = threading.Lock()  # one job per host at a time

    def remote_command(self, req: JobRequest, argv: list[str], job_dir: str) -> str:
        env = " ".join(f"{k}={shlex.quote(v)}" for k, v in sorted(req.env_vars.items()))
        cmd = " ".join(shlex.quote(a) for a in argv)
        d = shlex.quote(job_dir)
        return (f"cd {shlex.quote(self.workdir)} && mkdir -p {d} && "
                f"{('env ' + env + ' ') if env else ''}{cmd} > {d}/job.log 2>&1")

    def submit(self, req: JobRequest) -> JobHandle:
        name = safe_job_suffix(req.name)
        local_dir = os.path.join(self.local_root, name)
        os.makedirs(local_dir, exist_ok=True)
        h = JobHandle(self, req, local_dir)
        h._set("PENDING")
        remote_dir = f"{self.remote_root}/{name}"

        def go():
            with self.lock:
                argv = _write_payload(req, local_dir)
                if req.entrypoint.command is None:  # ship the pickled entry point
                    self.runner.run(f"mkdir -p {shlex.quote(remote_dir)}")
                    self.runner.put(os.path.join(local_dir, "entry.pkl"), f"{remote_dir}/entry.pkl")
                    argv = [self.python, "-m", "marin_experiments_b200.cluster", "run", f"{remote_dir}/entry.pkl"]
                argv = _job_argv(req, argv, 29800) if argv[0] == sys.executable else argv
                cmd = self.remote_command(req, argv, remote_dir)
                while True:
                    h.attempts += 1
                    h._set("RUNNING")
                    code = self.runner.run(cmd, timeout=req.timeout_s)
                    if code == 0:
                        h._set("SUCCEEDED", 0)
                        return
                    if h.attempts > req.max_retries_failure:
                        h._set("FAILED", code)
                        return

        threading.Thread(target=go, daemon=True).start()
        return h

    def _cancel(self, h: JobHandle) -> None:
        h._set("KILLED", None)


# ------------------------------------------------------------------------------- entry points
_CLIENT = None


def current_client():
    """The client named by ``MXK_CLUSTER``: ``local`` (default) or ``ssh://[user@]host[:port]``
    (``MXK_CLUSTER_WORKDIR`` is the remote checkout)."""
    global _CLIENT
    if _CLIENT is None:
        spec = os.environ.get("MXK_CLUSTER", "local")
        if spec == "local":
            _CLIENT = LocalClient(os.environ.get("MXK_JOBS_DIR", "jobs"))
        elif spec.startswith("ssh://"):
            m = re.match(r"ssh://(?:([^@]+)@)?([^:/]+)(?::(\d+))?", spec)
            if not m:
                raise ValueError(f"bad MXK_CLUSTER {spec!r}")
            _CLIENT = SSHClient(ParamikoRunner(m.group(2), m.group(1), int(m.group(3) or 22)),
                                workdir=os.environ.get("MXK_CLUSTER_WORKDIR", "."))
        else:
            raise ValueError(f"unknown MXK_CLUSTER {spec!r}")
    return _CLIENT


def set_client(client) -> None:
    global _CLIENT
    _CLIENT = client


def dispatch_grug_training_run(*, run_id: str, config, local_entrypoint: Callable, resources: ResourceConfig,
                               max_retries_failure: int = 3, client=None, timeout_s: float | None = None) -> JobHandle:
    """Submit ``local_entrypoint(config)`` as job ``grug-train-<run_id>`` with the forwarded runtime
    environment and wait for it (raises ``JobFailed`` when its retries are exhausted)."""
    req = JobRequest(name=f"grug-train-{safe_job_suffix(run_id)}",
                     entrypoint=Entrypoint.from_callable(local_entrypoint, args=[config]),
                     resources=resources, env_vars=forwarded_env_vars(), max_retries_failure=max_retries_failure,
                     timeout_s=timeout_s)
    job = (client or current_client()).submit(req)
    job.wait(raise_on_failure=True)
    return job


def _run_pickled(path: str) -> None:
    import cloudpickle

    with open(path, "rb") as f:
        fn, args, kwargs = cloudpickle.load(f)
    fn(*args, **kwargs)


if __name__ == "__main__":
    if len(sys.argv) == 3 and sys.argv[1] == "run":
        _run_pickled(sys.argv[2])
    else:
        sys.exit("usage: python -m marin_experiments_b200.cluster run <entry.pkl>")
