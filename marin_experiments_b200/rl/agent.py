"""Terminal agent loop and sandbox (openthoughts-agent/eval/sandbox.py:36-379,
openthoughts-agent/rl/environment.py:41-123, openthoughts-agent/training/agent_sft.py:39-307).

``LocalSandbox`` runs shell commands in a private temporary working directory with a hard timeout
and resource limits (CPU seconds, address space, file size, process count) set in the child before
``exec``. ``NamespaceSandbox`` adds kernel namespaces through ``unshare``: a network namespace with
no interfaces up (no network at all, loopback included), its own PID namespace with a fresh
``/proc`` (the command is PID 1 and sees no host processes), and private IPC and host-name
namespaces -- the isolation the reference gets from a gVisor (runsc) container, short of a
separate kernel. ``make_sandbox()`` picks the namespace sandbox when ``unshare`` works on the host
and falls back to the process-level one otherwise.

``run_episode`` drives a policy (any ``generate(prompt) -> str``): the reply's command (between
``<cmd>`` and ``</cmd>``) is executed, its output is appended as a tool turn, until the reply
contains ``<done/>`` or the turn budget ends; a task's checker scores the final sandbox state. Conversations are kept as ChatML messages, so episodes can be replayed as SFT data
(``data.chat.encode_chat`` masks the assistant turns).
"""

from __future__ import annotations

import os
import re
import resource
import shutil
import subprocess
import tempfile
from collections.abc import Callable
from dataclasses import dataclass, field


@dataclass
class ExecResult:
    stdout: str
    stderr: str
    exit_code: int
    timed_out: bool = False


class LocalSandbox:
    def __init__(self, cpu_s: int = 10, mem_mb: int = 1024, fsize_mb: int = 64, nproc: int = 64):
        self.dir = tempfile.mkdtemp(prefix="mxk-sandbox-")
        self.limits = (cpu_s, mem_mb, fsize_mb, nproc)

    def _preexec(self):
        cpu, mem, fs, npr = self.limits
        resource.setrlimit(resource.RLIMIT_CPU, (cpu, cpu))
        resource.setrlimit(resource.RLIMIT_AS, (mem << 20, mem << 20))
        resource.setrlimit(resource.RLIMIT_FSIZE, (fs << 20, fs << 20))
        resource.setrlimit(resource.RLIMIT_NPROC, (npr, npr))
        os.setsid()

    def exec(self, command: str, *, timeout: float = 30.0) -> ExecResult:
        env = {"PATH": "/usr/bin:/bin", "HOME": self.dir, "LANG": "C.UTF-8"}
        try:
            p = subprocess.run(["/bin/bash", "-c", command], cwd=self.dir, env=env, capture_output=True, text=True,
                               timeout=timeout, preexec_fn=self._preexec)
            return ExecResult(p.stdout, p.stderr, p.returncode)
        except subprocess.TimeoutExpired as e:
            return ExecResult(e.stdout or "", (e.stderr or "") + "\n[timeout]", 124, timed_out=True)

    def close(self):
        shutil.rmtree(self.dir, ignore_errors=True)


class NamespaceSandbox(LocalSandbox):
    """``LocalSandbox`` inside fresh network / PID / mount / IPC / UTS namespaces (a user namespace
    too when not running as root, so no privilege is needed)."""

    def __init__(self, network: bool = False, **limits):
        super().__init__(**limits)
        self.network = network

    def _prefix(self) -> list[str]:
        # --kill-child: a timed-out command's namespace init dies with unshare, and the kernel then
        # ends every process left in the namespace
        cmd = ["unshare", "--pid", "--fork", "--kill-child", "--mount-proc", "--ipc", "--uts"]
        if not self.network:
            cmd.append("--net")
        if os.geteuid() != 0:
            cmd += ["--user", "--map-root-user"]
        return cmd

    def exec(self, command: str, *, timeout: float = 30.0) -> ExecResult:
        env = {"PATH": "/usr/bin:/bin", "HOME": self.dir, "LANG": "C.UTF-8"}
        try:
            p = subprocess.run(self._prefix() + ["/bin/bash", "-c", command], cwd=self.dir, env=env,
                               capture_output=True, text=True, timeout=timeout, preexec_fn=self._preexec)
            return ExecResult(p.stdout, p.stderr, p.returncode)
        except subprocess.TimeoutExpired as e:
            return ExecResult(e.stdout or "", (e.stderr or "") + "\n[timeout]", 124, timed_out=True)


_NS_OK: bool | None = None


def namespaces_available() -> bool:
    global _NS_OK
    if _NS_OK is None:
        try:
            sb = NamespaceSandbox()
            try:
                _NS_OK = sb.exec("echo $$", timeout=10).stdout.strip() == "1"
            finally:
                sb.close()
        except (OSError, subprocess.SubprocessError):
            _NS_OK = False
    return _NS_OK


def make_sandbox(kind: str = "auto", **kw) -> LocalSandbox:
    """``"namespace"``, ``"local"`` or ``"auto"`` (namespaces when the host allows them)."""
    if kind == "namespace" or (kind == "auto" and namespaces_available()):
        return NamespaceSandbox(**kw)
    if kind in ("local", "auto"):
        return LocalSandbox(**kw)
    raise ValueError(f"unknown sandbox kind {kind!r}")


@dataclass
class AgentTask:
    instruction: str
    check: Callable[[LocalSandbox], float]
    setup: str | None = None


@dataclass
class Episode:
    messages: list = field(default_factory=list)
    reward: float = 0.0
    turns: int = 0


SYSTEM = ("You operate a Linux shell. Reply with one command as <cmd>...</cmd>; you will see its output. "
          "Reply <done/> when the task is complete.")
_CMD = re.compile(r"<cmd>(.*?)</cmd>", re.S)


def run_episode(policy: Callable[[list], str], task: AgentTask, max_turns: int = 8, timeout: float = 30.0,
                sandbox: str = "auto") -> Episode:
    sb = make_sandbox(sandbox)
    ep = Episode(messages=[{"role": "system", "content": SYSTEM}, {"role": "user", "content": task.instruction}])
    try:
        if task.setup:
            sb.exec(task.setup, timeout=timeout)
        for _ in range(max_turns):
            reply = policy(ep.messages)
            ep.messages.append({"role": "assistant", "content": reply})
            ep.turns += 1
            m = _CMD.search(reply)
            if m:
                r = sb.exec(m.group(1).strip(), timeout=timeout)
                out = (r.stdout + r.stderr)[-4000:]
                ep.messages.append({"role": "tool", "content": f"[exit {r.exit_code}]\n{out}"})
            if "<done/>" in reply or not m:
                break
        ep.reward = float(task.check(sb))
    finally:
        sb.close()
    return ep
