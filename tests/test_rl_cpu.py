"""GRPO / Dr.GRPO objectives, environments, the safe program interpreter and a learner step."""

import pytest
import torch

from marin_experiments_b200.rl.envs import CalculatorEnv, CodingEnv, ProgramError, run_program
from marin_experiments_b200.rl.grpo import group_advantages, policy_loss


def test_advantages():
    r = torch.tensor([1.0, 0.0, 0.0, 1.0, 0.5, 0.5, 0.5, 0.5])
    dr = group_advantages(r, 4, "dr_grpo")
    assert torch.allclose(dr[:4], torch.tensor([0.5, -0.5, -0.5, 0.5])) and torch.all(dr[4:] == 0)
    g = group_advantages(r, 4, "grpo")
    assert torch.allclose(g[:4], torch.tensor([1.0, -1.0, -1.0, 1.0]), atol=1e-4)


def test_policy_loss_gradient_direction():
    logp = torch.zeros(2, 3, requires_grad=True)
    mask = torch.ones(2, 3)
    loss, _ = policy_loss(logp, mask, torch.tensor([1.0, -1.0]))
    loss.backward()
    assert torch.all(logp.grad[0] < 0) and torch.all(logp.grad[1] > 0)  # raise good, lower bad


def test_envs_and_interpreter():
    env = CalculatorEnv(seed=1)
    t = env.sample()
    assert env.reward(f"the answer is {t.answer}", t.answer) == 1.0
    assert 0 <= env.reward("123", t.answer) < 1.0
    assert run_program("s = 0\nfor i in range(5):\n    s += i\nprint(s)") == "10"
    assert run_program("x = 3\nwhile x > 0:\n    print(x)\n    x -= 1") == "3\n2\n1"
    with pytest.raises(ProgramError):
        run_program("import os")
    with pytest.raises(ProgramError):
        run_program("while True:\n    pass", max_steps=100)
    assert CodingEnv.reward("print(17 + 25)\nEND junk", "42") == 1.0
    assert CodingEnv.reward("open('x')", "42") == 0.0


def test_learner_step_updates_policy():
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from marin_experiments_b200.rl.learner import GRPOConfig, GRPOLearner

    cfg = Qwen3Config(vocab_size=257, hidden_dim=64, intermediate_dim=128, num_layers=1, num_heads=2, num_kv_heads=1,
                      head_dim=32, max_seq_len=128)
    m = Qwen3Model(cfg).init_weights(0)
    before = m.w_qkv if hasattr(m, "w_qkv") else m.layers[0].w_q.detach().clone()
    lr = GRPOLearner(m, ByteTokenizer(), CalculatorEnv(seed=0), GRPOConfig(group_size=4, max_new_tokens=6, lr=1e-2))
    met = lr.step(n_prompts=2)
    assert set(met) >= {"loss", "reward_mean", "grad_norm"}
    assert not torch.equal(before, m.layers[0].w_q.detach())


def test_agent_episode_in_sandbox():
    import os

    from marin_experiments_b200.rl.agent import AgentTask, LocalSandbox, run_episode

    sb = LocalSandbox()
    r = sb.exec("echo hi > a.txt && cat a.txt")
    assert r.stdout.strip() == "hi" and r.exit_code == 0
    assert sb.exec("sleep 5", timeout=0.5).timed_out
    sb.close()
    task = AgentTask("create f.txt containing 42",
                     check=lambda s: float(open(os.path.join(s.dir, "f.txt")).read().strip() == "42"))
    script = iter(["<cmd>echo 42 > f.txt</cmd>", "<done/>"])
    ep = run_episode(lambda msgs: next(script), task)
    assert ep.reward == 1.0 and ep.turns == 2
    assert [m["role"] for m in ep.messages] == ["system", "user", "assistant", "tool", "assistant"]


def test_namespace_sandbox_isolation():
    from marin_experiments_b200.rl import agent

    if not agent.namespaces_available():
        import pytest

        pytest.skip("unshare is not permitted on this host")
    sb = agent.make_sandbox("auto")
    try:
        assert isinstance(sb, agent.NamespaceSandbox)
        assert sb.exec("echo $$").stdout.strip() == "1"  # own PID namespace
        assert sb.exec("ps -e --no-headers | wc -l").stdout.strip() in ("2", "3")  # bash, ps (, wc)
        r = sb.exec("python3 -c \"import socket; socket.create_connection(('1.1.1.1', 53), 2)\"", timeout=20)
        assert r.exit_code != 0 and "unreachable" in r.stderr.lower()
        assert sb.exec("echo x > f && cat f").stdout.strip() == "x"  # working directory persists
        assert sb.exec("sleep 30 & sleep 30", timeout=0.5).timed_out
    finally:
        sb.close()


def test_toy_grpo_learns():
    from marin_experiments_b200.rl.toy import train_toy

    r = train_toy(steps=25)
    assert r.first < 0.45 and r.last > 0.8, r.rewards


def test_learner_with_engine_rollouts():
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from marin_experiments_b200.rl.learner import GRPOConfig, GRPOLearner
    from marin_experiments_b200.serving.engine import Engine, SamplingParams

    cfg = Qwen3Config(vocab_size=257, hidden_dim=64, intermediate_dim=128, num_layers=1, num_heads=2, num_kv_heads=1,
                      head_dim=32, max_seq_len=128)
    m = Qwen3Model(cfg).init_weights(0)
    tok = ByteTokenizer()
    eng = Engine(m, tok, max_batch=4)
    ids = eng.generate_ids([tok.encode("12+3="), tok.encode("ab")], SamplingParams(max_tokens=5, temperature=0.0))
    assert [tok.decode(x) for x in ids] == eng.generate(["12+3=", "ab"], max_tokens=5, temperature=0.0)
    before = m.layers[0].w_q.detach().clone()
    lr = GRPOLearner(m, tok, CalculatorEnv(seed=0),
                     GRPOConfig(group_size=4, max_new_tokens=6, lr=1e-2, use_engine=True))
    met = lr.step(n_prompts=2)
    assert torch.isfinite(torch.tensor(met["loss"])) and lr.engine is not None
    assert not torch.equal(before, m.layers[0].w_q.detach())
    lr.step(n_prompts=1)  # the engine is reused (weights refreshed in place)
