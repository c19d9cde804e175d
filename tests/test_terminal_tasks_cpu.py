"""Built-in terminal tasks: every family solved by its oracle and failed by a do-nothing agent; the
ChatML adapter for multi-turn GRPO; oracle SFT transcripts; the agent ladder stage."""

import json

import pytest
import torch

from marin_experiments_b200.data.chat import IM_END, IM_START
from marin_experiments_b200.rl import pipeline, terminal, terminal_tasks


@pytest.fixture(scope="module")
def tasks(tmp_path_factory):
    root = str(tmp_path_factory.mktemp("tasks"))
    terminal_tasks.write_tasks(root, 2 * terminal_tasks.FAMILIES, seed=5)
    return terminal.load_tasks(root)


def test_oracle_solves_and_idle_fails(tasks):
    acts = {t.task_id: terminal_tasks.oracle_actions(t) for t in tasks}

    def oracle(msgs):
        task_text = msgs[0]["content"]
        t = next(x for x in tasks if x.instruction in task_text)
        return acts[t.task_id][sum(m["role"] == "assistant" for m in msgs)]

    res = terminal.evaluate(oracle, tasks, max_turns=4, sandbox="local")
    assert res["solved"] == len(tasks) and res["parse_failures"] == 0
    idle = json.dumps({"analysis": "", "plan": "", "commands": [], "task_complete": True})
    res0 = terminal.evaluate(lambda m: idle, tasks, max_turns=2, sandbox="local")
    assert res0["solved"] == 0


def test_chat_adapter_and_transcript(tasks):
    t = tasks[0]
    env = terminal.ChatTerminalEnv(t, max_turns=4, sandbox="local")
    assert env.render().startswith(f"{IM_START}user\n") and env.render().endswith(f"{IM_START}assistant\n")
    run, done = terminal_tasks.oracle_actions(t)
    assert not env.step(run + IM_END + "junk after the end marker")
    fb = env.feedback
    assert fb.startswith(f"{IM_START}user\nNew terminal output:") and fb.endswith(f"{IM_START}assistant\n")
    assert env.step(done + IM_END) and env.feedback is None
    assert env.reward() == 1.0 and env.reward() == 1.0  # graded once, then cached
    segs = pipeline.agent_transcript(t, sandbox="local")
    assert [m for _, m in segs] == [0, 1, 0, 1]
    assert [s for s, m in segs if m] == [run + IM_END, done + IM_END]
    assert segs[2][0].startswith(f"\n{IM_START}user\nNew terminal output:")


def test_agent_stage_runs(tmp_path, monkeypatch):
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model

    tiny = {"agent": [pipeline.Stage("sft_grpo", 2, sft_steps=1, grpo_steps=1, group_size=2, prompts_per_step=1,
                                     kind="agent")]}
    monkeypatch.setattr(pipeline, "EXPERIMENTS", tiny)
    cfg = Qwen3Config(vocab_size=257, hidden_dim=64, intermediate_dim=128, num_layers=1, num_heads=2, num_kv_heads=1,
                      head_dim=32, max_seq_len=4096)
    res = pipeline.run("agent", lambda: Qwen3Model(cfg).init_weights(0), ByteTokenizer(), str(tmp_path / "res"),
                       max_program_tokens=6, seq_len=2048, eval_tools=2, sandbox="local",
                       task_root=str(tmp_path / "tasks"), agent_turns=2)["sft_grpo"]
    assert res["eval"]["total"] == 2 and res["eval"]["solved"] == 0 and "grpo" in res
    assert torch.isfinite(torch.tensor(res["sft"]["last_loss"]))
