"""RL curriculum (fixed cadence + mastery gate) and the test-case-graded coding environment."""

import random

import pytest

from marin_experiments_b200.rl.curriculum import (Curriculum, CurriculumConfig, TestCaseEnv, evaluate_passk,
                                                  pass_at_k)


def test_mastery_gate_and_fallback():
    cur = Curriculum(CurriculumConfig(num_levels=3, steps_per_level=4, max_holds=2))
    assert cur.weights() == [1.0, 0.0, 0.0]
    for _ in range(4):  # level 1 mastered: unlocks level 2 at the window end
        cur.record(1, 1.0)
        cur.on_step()
    assert cur.unlocked == 2
    unlocked_at = []
    for s in range(12):  # level 2 never succeeds: hold 2 windows, then advance anyway
        cur.record(2, 0.0)
        if cur.on_step():
            unlocked_at.append(cur.step)
    assert unlocked_at == [16] and cur.unlocked == 3
    for _ in range(8):
        cur.on_step()
    assert cur.unlocked == 3  # no level past the last


def test_sampling_frontier_floor_and_graduation():
    cfg = CurriculumConfig(num_levels=4, frontier_weight=0.6, floor_weight=0.05)
    cur = Curriculum(cfg)
    cur.unlocked = 3
    w = cur.weights()
    assert w[3] == 0.0 and abs(sum(w) - 1.0) < 1e-12 and w[2] > w[0] == w[1]
    cur.record(1, 1.0)  # level 1 graduated -> floor
    w2 = cur.weights()
    assert w2[0] < w[0] and w2[0] >= 0.05 / sum([0.05, 0.2, 0.6]) - 1e-12
    rng = random.Random(0)
    levels = [cur.sample_level(rng) for _ in range(2000)]
    assert set(levels) <= {1, 2, 3} and levels.count(3) > levels.count(2) > levels.count(1)
    st = cur.state_dict()
    other = Curriculum(cfg)
    other.load_state_dict(st)
    assert other.state_dict() == st


def test_testcase_env_rewards_and_held_out():
    env = TestCaseEnv(seed=1)
    for level in range(1, 6):
        p = env.sample(level)
        assert len(p.tests) == 5 and f"Level {level}" in p.prompt
        assert env.reward(p.reference + "\nEND trailing text", p) == 1.0
        assert env.reward("print(0)", p) < 1.0
        assert env.reward("this is not a program", p) == 0.0
    # partial credit: right for some inputs only
    p = env.sample(3)
    partial = "if n < 10:\n    print(n * (n + 1) // 2)\nelse:\n    print(0)"
    r = env.reward(partial, p)
    want = sum(int(pre.split("=")[1]) < 10 for pre, _ in p.tests) / 5
    assert r == pytest.approx(want)
    a, b = env.held_out(2, 3), env.held_out(2, 3)
    assert [x.tests for x in a] == [x.tests for x in b]


def test_pass_at_k():
    assert pass_at_k(10, 0, 1) == 0.0 and pass_at_k(10, 10, 3) == 1.0
    assert pass_at_k(10, 3, 1) == pytest.approx(0.3)
    assert pass_at_k(4, 1, 2) == pytest.approx(0.5)
    env = TestCaseEnv(seed=2)
    probs = env.held_out(1, 4) + env.held_out(3, 4)
    res = evaluate_passk(lambda p: [p.reference, "print(1)", "print(2)", "x"], probs, k=2)
    assert set(res) == {1, 3} and all(v == pytest.approx(0.5) for v in res.values())


def test_curriculum_task_source_feeds_the_schedule():
    from marin_experiments_b200.rl.curriculum import CurriculumTaskSource

    src = CurriculumTaskSource(TestCaseEnv(seed=3), Curriculum(CurriculumConfig(num_levels=5, steps_per_level=2)))
    for _ in range(2):
        tasks = [src.sample() for _ in range(3)]
        assert all(t.answer.level == 1 for t in tasks)
        for t in tasks:
            assert src.reward(t.answer.reference, t.answer) == 1.0
        src.on_step()
    assert src.cur.unlocked == 2 and src.cur.ema[0] == 1.0
