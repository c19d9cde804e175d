"""Terminal-task agents: task directories, a JSON-action agent loop, test-script grading, the
reset / step environment for RL and the agent-trace SFT data (openthoughts-agent/eval/tb_tasks.py,
openthoughts-agent/eval/agent_loop.py, openthoughts-agent/eval/grade.py,
openthoughts-agent/rl/environment.py, openthoughts-agent/agent_data/agent_traces.py).

A task is a directory::

    <task id>/instruction.md        the prompt
    <task id>/task.toml             optional: [agent] timeout_sec, [verifier] timeout_sec
    <task id>/environment/...       files the agent starts with (a Dockerfile there is not built:
                                    there is no container runtime, the sandbox is a directory)
    <task id>/tests/test.sh         the grader; writes a score in [0, 1] to reward.txt
    <task id>/solution/solve.sh     the oracle (never shown to the agent)

Each assistant turn is a JSON object ``{"analysis", "plan", "commands": [{"keystrokes",
"duration"}], "task_complete"}``; prose around it is tolerated (the last balanced object with a
``commands`` key is taken). The commands' keystrokes run in the sandbox (``rl.agent.make_sandbox``:
namespaces where the host allows them) and the terminal output comes back as the next user turn;
an unparsable turn gets a corrective message instead. The episode ends when the agent marks the
task complete with no commands left, or after ``max_turns``. Grading copies ``tests/`` into the
sandbox, runs ``tests/test.sh`` under the verifier timeout and reads ``reward.txt`` (the first of
``logs/verifier/reward.txt``, ``tests/reward.txt``, ``reward.txt`` that exists; any such file the agent
wrote is deleted before the grader runs); without one the script's exit status decides (0 -> 1.0). Solved means score >= 1. ``ChatTerminalEnv`` presents the
same loop as ChatML text to the multi-turn GRPO learner.
"""

from __future__ import annotations

import json
import os
import shutil
import tomllib
from collections.abc import Callable
from dataclasses import dataclass, field

from .agent import LocalSandbox, make_sandbox

SYSTEM_PROMPT = (
    "You solve tasks in a Linux shell. Each reply is one JSON object:\n"
    '{"analysis": "what the terminal shows and what is left to do", "plan": "the next steps", '
    '"commands": [{"keystrokes": "ls -la\\n", "duration": 0.1}], "task_complete": false}\n'
    "The keystrokes run in order; you then see the new terminal output. Set task_complete to true, "
    "with an empty commands list, only when the task is done."
)
PARSE_FAIL = "Your reply could not be parsed as a JSON action with a commands list. Reply with one JSON object."
_REWARD_FILES = ("logs/verifier/reward.txt", "tests/reward.txt", "reward.txt")
MAX_OBSERVATION = 8000


@dataclass(frozen=True)
class Action:
    analysis: str
    plan: str
    commands: list
    task_complete: bool
    ok: bool


def _objects(text: str):
    """Balanced ``{...}`` spans of ``text`` outside string literals, in order."""
    depth, start, in_str, esc = 0, -1, False, False
    for i, ch in enumerate(text):
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
            continue
        if ch == '"' and depth > 0:
            in_str = True
        elif ch == "{":
            if depth == 0:
                start = i
            depth += 1
        elif ch == "}" and depth > 0:
            depth -= 1
            if depth == 0:
                yield text[start:i + 1]


def parse_action(text: str) -> Action:
    best = None
    for span in _objects(text or ""):
        try:
            obj = json.loads(span)
        except json.JSONDecodeError:
            continue
        if isinstance(obj, dict) and isinstance(obj.get("commands"), list):
            best = obj
    if best is None:
        return Action("", "", [], False, False)
    cmds = [c for c in best["commands"] if isinstance(c, dict) and isinstance(c.get("keystrokes"), str)]
    return Action(str(best.get("analysis", "")), str(best.get("plan", "")), cmds, bool(best.get("task_complete")),
                  True)


def format_observation(output: str, limit: int = MAX_OBSERVATION) -> str:
    if len(output) > limit:
        output = f"[... {len(output) - limit} characters cut ...]\n" + output[-limit:]
    return f"New terminal output:\n{output}"


@dataclass(frozen=True)
class TerminalTask:
    task_id: str
    root: str
    instruction: str
    agent_timeout_s: float = 600.0
    verifier_timeout_s: float = 300.0
    meta: dict = field(default_factory=dict)


def load_task(path: str) -> TerminalTask:
    with open(os.path.join(path, "instruction.md")) as f:
        instruction = f.read().strip()
    meta: dict = {}
    toml = os.path.join(path, "task.toml")
    if os.path.exists(toml):
        with open(toml, "rb") as f:
            meta = tomllib.load(f)
    return TerminalTask(os.path.basename(os.path.normpath(path)), path, instruction,
                        float(meta.get("agent", {}).get("timeout_sec", 600.0)),
                        float(meta.get("verifier", {}).get("timeout_sec", 300.0)), meta)


def load_tasks(root: str) -> list[TerminalTask]:
    """Every ``<root>/<task id>/`` with an ``instruction.md``, sorted by id."""
    return [load_task(os.path.join(root, d)) for d in sorted(os.listdir(root))
            if os.path.isfile(os.path.join(root, d, "instruction.md"))]


def prepare(sb: LocalSandbox, task: TerminalTask) -> None:
    env = os.path.join(task.root, "environment")
    if os.path.isdir(env):
        shutil.copytree(env, sb.dir, dirs_exist_ok=True, ignore=shutil.ignore_patterns("Dockerfile"))


@dataclass(frozen=True)
class GradeResult:
    task_id: str
    solved: bool
    score: float
    exit_code: int
    detail: str


def grade(sb: LocalSandbox, task: TerminalTask) -> GradeResult:
    # a score file the agent left behind must not count: only what the grader writes now does
    for rel in _REWARD_FILES:
        p = os.path.join(sb.dir, rel)
        if os.path.lexists(p):
            if os.path.isdir(p) and not os.path.islink(p):
                shutil.rmtree(p)
            else:
                os.remove(p)
    # the grader's files replace whatever the agent put at tests/ (a link there, or a link inside it,
    # would otherwise send the copy outside the sandbox)
    tdir = os.path.join(sb.dir, "tests")
    if os.path.isdir(tdir) and not os.path.islink(tdir):
        shutil.rmtree(tdir)
    elif os.path.lexists(tdir):
        os.remove(tdir)
    shutil.copytree(os.path.join(task.root, "tests"), tdir)
    r = sb.exec("bash tests/test.sh", timeout=task.verifier_timeout_s)
    score = None
    for rel in _REWARD_FILES:
        p = os.path.join(sb.dir, rel)
        if os.path.exists(p):
            try:
                score = max(0.0, min(1.0, float(open(p).read().strip().split()[0])))
            except (ValueError, IndexError):
                score = 0.0
            break
    if score is None:
        score = 1.0 if r.exit_code == 0 and not r.timed_out else 0.0
    return GradeResult(task.task_id, score >= 1.0, score, r.exit_code, (r.stdout + r.stderr)[-2000:])


@dataclass
class TerminalEpisode:
    messages: list
    turns: int = 0
    parse_failures: int = 0
    grade: GradeResult | None = None

    @property
    def reward(self) -> float:
        return self.grade.score if self.grade else 0.0


class TerminalEnv:
    """``reset(task) -> messages``, ``step(reply) -> (observation | None, done)``, ``final_reward()``:
    the loop for a rollout engine; every step's reward is 0 and the graded score is the terminal
    reward."""

    def __init__(self, max_turns: int = 16, sandbox: str = "auto", command_timeout_s: float = 60.0):
        self.max_turns, self.kind, self.command_timeout_s = max_turns, sandbox, command_timeout_s
        self.sb: LocalSandbox | None = None
        self.task: TerminalTask | None = None
        self.episode: TerminalEpisode | None = None

    def reset(self, task: TerminalTask) -> list:
        self.close()
        self.sb, self.task = make_sandbox(self.kind), task
        prepare(self.sb, task)
        self.episode = TerminalEpisode([{"role": "user", "content": f"{SYSTEM_PROMPT}\n\nTask:\n{task.instruction}"}])
        return self.episode.messages

    def step(self, reply: str) -> tuple[str | None, bool]:
        ep = self.episode
        ep.messages.append({"role": "assistant", "content": reply})
        ep.turns += 1
        act = parse_action(reply)
        if not act.ok:
            ep.parse_failures += 1
            obs = PARSE_FAIL
        elif act.task_complete and not act.commands:
            return None, True
        else:
            keys = "".join(c["keystrokes"] for c in act.commands)
            r = self.sb.exec(keys, timeout=self.command_timeout_s)
            obs = format_observation(r.stdout + r.stderr + ("\n[timed out]" if r.timed_out else ""))
        done = ep.turns >= self.max_turns
        if not done:
            ep.messages.append({"role": "user", "content": obs})
        return (None if done else obs), done

    def final_reward(self) -> float:
        self.episode.grade = grade(self.sb, self.task)
        return self.episode.grade.score

    def close(self) -> None:
        if self.sb is not None:
            self.sb.close()
            self.sb = None


def run_episode(model_fn: Callable[[list], str], task: TerminalTask, max_turns: int = 16,
                sandbox: str = "auto") -> TerminalEpisode:
    env = TerminalEnv(max_turns, sandbox)
    try:
        msgs = env.reset(task)
        done = False
        while not done:
            _, done = env.step(model_fn(msgs))
        env.final_reward()
        return env.episode
    finally:
        env.close()


def evaluate(model_fn: Callable[[list], str], tasks: list[TerminalTask], max_turns: int = 16,
             sandbox: str = "auto") -> dict:
    eps = [run_episode(model_fn, t, max_turns, sandbox) for t in tasks]
    n = max(len(eps), 1)
    return {"solved": sum(e.grade.solved for e in eps), "total": len(eps),
            "mean_score": sum(e.reward for e in eps) / n, "mean_turns": sum(e.turns for e in eps) / n,
            "parse_failures": sum(e.parse_failures for e in eps), "episodes": eps}


def load_agent_traces(path: str, limit: int | None = None):
    """Agent SFT traces (``conversations`` of user / assistant turns, plus metadata columns) from a
    local Parquet or JSON-lines file, as ``{"messages", "metadata"}`` rows for the chat cache."""
    from ..data.instruct import Adapter, DatasetSpec, _read_file, transform_row

    spec = DatasetSpec("traces", "", Adapter(conversation_column="conversations", replacements=()),
                       ("agent", "model", "task", "episode", "run_id", "trial_name"))
    n = 0
    for row in _read_file(path):
        out = transform_row(row, spec)
        if out is None:
            continue
        yield out
        n += 1
        if limit is not None and n >= limit:
            return


class ChatTerminalEnv:
    """``TerminalEnv`` as text for ``rl.multiturn.MultiTurnGRPO``: ``render()`` is the ChatML of the
    opening turn ending in an open assistant header, an assistant turn is what the policy writes up
    to ``<|im_end|>``, ``feedback`` is the next user turn (the terminal output) plus a fresh
    assistant header, and ``reward()`` grades the sandbox once and closes it."""

    def __init__(self, task: TerminalTask, max_turns: int = 8, sandbox: str = "auto"):
        from ..data.chat import IM_END, IM_START, render_chatml

        self._im = (IM_START, IM_END)
        self._render = render_chatml
        self.env = TerminalEnv(max_turns, sandbox)
        self.env.reset(task)
        self._obs: str | None = None
        self.done = False
        self._reward: float | None = None

    def render(self) -> str:
        return self._render(self.env.episode.messages[:1], add_generation_prompt=True)

    def step(self, text: str) -> bool:
        reply = text.split(self._im[1], 1)[0].strip()
        self._obs, self.done = self.env.step(reply)
        return self.done

    @property
    def feedback(self) -> str | None:
        if self.done or self._obs is None:
            return None
        s, e = self._im
        return f"{s}user\n{self._obs}{e}\n{s}assistant\n"

    def reward(self) -> float:
        if self._reward is None:
            try:
                self._reward = self.env.final_reward()
            finally:
                self.env.close()
        return self._reward
