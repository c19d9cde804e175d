"""Tool-calling chains, the write-run-revise coding agent and the multi-turn GRPO learner."""

import random

import torch

from marin_experiments_b200.rl import code_agent as ca
from marin_experiments_b200.rl import tools


def _calc_policy(wrong_first: bool = False):
    """Scripted policy for chain tasks: calls CALC on the next operand pair, then answers."""

    def policy(text: str) -> str:
        q = [ln for ln in text.split("\n") if ln.startswith("Q: ")][-1]
        ops = [int(v) for v in q[3:].split(" * ")]
        tail = text.split(q, 1)[1]
        results = [int(ln.split(": ")[1]) for ln in tail.split("\n") if ln.startswith("Tool result: ")]
        if not results:
            a = ops[0] + (1 if wrong_first else 0)
            return f"CALC({a} * {ops[1]})\n"
        if len(results) < len(ops) - 1:
            return f"CALC({results[-1]} * {ops[len(results) + 1]})\n"
        return f"{results[-1]}\n"

    return policy


def test_chain_tasks_and_rewards():
    ts = tools.chain_tasks(20, seed=3, depth=2)
    assert ts == tools.chain_tasks(20, seed=3, depth=2) and all(t.depth == 2 for t in ts)
    t = ts[0]
    assert int(t.answer) == t.operands[0] * t.operands[1] * t.operands[2]
    env = tools.rollout(_calc_policy(), t)
    assert env.calls == 2 and env.final_answer == t.answer
    assert abs(tools.total_reward(env) - 1.9) < 1e-9 and abs(tools.total_reward(env, with_format=True) - 2.0) < 1e-9
    bad = tools.rollout(_calc_policy(wrong_first=True), t)
    # wrong first operand: the final answer copies the last tool result (+0.4) but misses the gold
    assert abs(tools.total_reward(bad) - 0.4) < 1e-9
    envs = [tools.rollout(_calc_policy(i % 2 == 1), x) for i, x in enumerate(ts)]
    m = tools.metrics(envs, [tools.total_reward(e) for e in envs])
    assert m["tool/tool_call_rate"] == 1.0 and m["tool/arg_acc"] == 0.5 and m["arithmetic/solve_ratio"] == 0.5


def test_call_parsing_and_budget():
    assert tools.parse_call("CALC(12 * 34") == (12, 34) and not tools.call_closed("CALC(12 * 34")
    assert tools.parse_call("x CALC( 5*6 ) y") == (5, 6) and tools.call_closed("CALC( 5*6 )")
    assert tools.parse_call("56") is None
    t = tools.chain_tasks(1, seed=0, depth=1)[0]
    env = tools.rollout(lambda _: "CALC(2 * 3)\n", t)  # calls forever: the budget ends the episode
    assert env.calls == 1 and sum(r == "assistant" for r, _ in env.turns) == 2 and env.reward() == 0.0
    assert env.feedback is None and "Tool result: 6" in env.render()


def _code_policy(fix: bool, bug_seed: int = 0):
    """Writes the task's solution; with ``fix``, first a planted bug, then the solution."""

    def policy(text: str) -> str:
        prompt = text.rsplit("Task: ", 1)[1].split("\n", 1)[0]
        task = next(t for t in TASKS if t.prompt == prompt)
        if fix and "Tool result:" not in text.rsplit("Task: ", 1)[1]:
            bug = ca.make_bug(random.Random(bug_seed), task)
            if bug is not None:
                return bug[0] + "\nEND\n"
        return "```\n" + task.solution + "\nEND\n"

    return policy


TASKS = ca.coding_tasks(24, seed=5)


def test_code_agent_first_and_best():
    direct = ca.evaluate_multiturn(_code_policy(False), TASKS)
    assert direct["first_solve"] == 1.0 and direct["best_solve"] == 1.0 and direct["mean_rounds"] == 1.0
    rep = ca.evaluate_multiturn(_code_policy(True), TASKS)
    assert rep["best_solve"] == 1.0 and rep["first_solve"] < 0.2 and rep["mean_rounds"] > 1.8
    for e in rep["envs"]:
        assert e.reward() >= ca.SOLVED and e.rewards[0] < 1.0
    wrong = ca.run_episode(lambda _: "print('nope')\nEND\n", TASKS[0], max_rounds=3)
    assert not wrong.solved and len(wrong.history) == 3 and wrong.reward() < 1.0
    assert wrong.history[0][1] == "nope"
    assert ca.extract_program("print(1)\nTool result: 1\nprint(2)") == "print(1)"
    assert ca.extract_program("```python\nprint(3)\n```\nEND") == "print(3)"


def test_code_agent_feedback_and_grades():
    env = ca.CodeAgentEnv(TASKS[0])
    env.step("x = 1 / 0\nprint(x)\nEND\nprint('after END is ignored')")
    assert env.history[0][1].startswith("Error: ") and "ZeroDivisionError" in env.history[0][1]
    assert abs(env.rewards[0] - ca.W_HAS_CODE) < 1e-9
    assert env.feedback.startswith("Tool result: Error:")
    env.step("y = 2\nEND")
    assert env.history[1][1] == "(no output)"
    g = ca.grade(ca.micropy.run("print('45')"), "print('45')", "46\n")
    assert g["ran"] == 1.0 and g["exact"] == 0.0 and 0.0 < g["partial"] < 1.0
    stopped = ca.CodeAgentEnv(TASKS[0])
    assert stopped.step("") and stopped.reward() == 0.0  # an empty turn ends the episode
    long = ca.feedback(ca.micropy.run("for i in range(500):\n  print(i)"), "x")
    assert long.endswith("...(truncated)") and len(long) <= ca.MAX_FEEDBACK + 20


def test_sft_transcripts_and_passk():
    rng = random.Random(0)
    segs = [ca.sft_transcript(rng, t, fix_prob=1.0) for t in TASKS]
    with_fix = [s for s in segs if len(s) == 4]
    assert len(with_fix) >= len(TASKS) - 2
    for s in with_fix:
        assert [m for _, m in s] == [0, 1, 0, 1] and s[2][0].startswith("Tool result: ")
    assert all(len(ca.sft_transcript(rng, t, fix_prob=0.0)) == 2 for t in TASKS)

    def sample(prompt, k):
        task = next(t for t in TASKS if f"Task: {t.prompt}\n" in prompt)
        return [task.solution + "\nEND"] * (k // 2) + ["print(0)\nEND"] * (k - k // 2)

    pk = ca.evaluate_passk(sample, TASKS[:6], 4)
    assert abs(pk["pass@1"] - 0.5) < 1e-9 and pk["pass@4"] == 1.0
    rp = ca.evaluate_repair_passk(sample, TASKS[:6], 4)
    assert rp["tasks"] >= 5 and abs(rp["repair_pass@1"] - 0.5) < 1e-9


def test_multiturn_grpo_step():
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from marin_experiments_b200.rl.multiturn import MultiTurnConfig, MultiTurnGRPO

    cfg = Qwen3Config(vocab_size=257, hidden_dim=64, intermediate_dim=128, num_layers=1, num_heads=2, num_kv_heads=1,
                      head_dim=32, max_seq_len=1024)
    m = Qwen3Model(cfg).init_weights(0)
    before = m.layers[0].w_q.detach().clone()
    tasks = iter(tools.chain_tasks(8, seed=1, depth=1))
    short = "CALC(x * y), then the result.\n"
    lr = MultiTurnGRPO(m, ByteTokenizer(), lambda: next(tasks), lambda t: tools.CalcToolEnv(t, system=short),
                       MultiTurnConfig(group_size=2, max_turn_tokens=6, lr=1e-2, max_total_tokens=96),
                       reward_fn=tools.total_reward)
    ids, mask, env = lr.rollout(tools.chain_tasks(1, seed=2, depth=1)[0])
    assert len(ids) == len(mask) and sum(mask) >= 1 and mask[0] == 0
    met = lr.step(n_prompts=2)
    assert set(met) >= {"loss", "reward_mean", "grad_norm", "turns_mean", "trained_tokens"}
    assert torch.isfinite(torch.tensor(met["loss"])) and met["trained_tokens"] > 0
    assert not torch.equal(before, m.layers[0].w_q.detach())


def test_multiturn_transcript_masks_feedback():
    """With a scripted model the transcript holds the sampled turns (mask 1) and tool results (mask 0)."""
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.rl.multiturn import MultiTurnConfig, MultiTurnGRPO

    tok = ByteTokenizer()
    task = tools.ChainTask("Q: 12 * 13", (12, 13), "156")
    script = tok.encode("CALC(12 * 13)\n156\n")

    class Scripted(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(torch.zeros(1))
            self.pos = 0

        def forward_logits(self, x):
            out = torch.full((x.shape[0], x.shape[1], 257), -1e4)
            out[:, -1, script[self.pos % len(script)]] = 1e4
            self.pos += 1
            return out + self.w

    lr = MultiTurnGRPO(Scripted(), tok, lambda: task, lambda t: tools.CalcToolEnv(t),
                       MultiTurnConfig(group_size=1, max_turn_tokens=20, temperature=1e-3),
                       reward_fn=tools.total_reward)
    ids, mask, env = lr.rollout(task)
    text = tok.decode(ids)
    assert text.endswith("CALC(12 * 13)\nTool result: 156\n156\n")
    trained = tok.decode([t for t, k in zip(ids, mask) if k])
    assert trained == "CALC(12 * 13)\n156\n" and abs(tools.total_reward(env) - 1.9) < 1e-9


def test_multiturn_grpo_with_engine_turns():
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from marin_experiments_b200.rl.multiturn import MultiTurnConfig, MultiTurnGRPO

    cfg = Qwen3Config(vocab_size=257, hidden_dim=64, intermediate_dim=128, num_layers=1, num_heads=2, num_kv_heads=1,
                      head_dim=32, max_seq_len=1024)
    m = Qwen3Model(cfg).init_weights(0)
    before = m.layers[0].w_q.detach().clone()
    tasks = iter(tools.chain_tasks(8, seed=1, depth=1))
    lr = MultiTurnGRPO(m, ByteTokenizer(), lambda: next(tasks),
                       lambda t: tools.CalcToolEnv(t, system="CALC(x * y), then the result.\n"),
                       MultiTurnConfig(group_size=2, max_turn_tokens=6, lr=1e-2, max_total_tokens=96, use_engine=True),
                       reward_fn=tools.total_reward)
    met = lr.step(n_prompts=2)
    assert lr.engine is not None and met["trained_tokens"] > 0 and torch.isfinite(torch.tensor(met["loss"]))
    assert not torch.equal(before, m.layers[0].w_q.detach())
