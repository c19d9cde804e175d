"""Nine levels of test-graded ``def solve`` problems: references against CPython, test make-up,
dense grading, feedback, and the curriculum source over them."""

import contextlib
import io
import random

import pytest

from marin_experiments_b200.rl import solve_problems as S
from marin_experiments_b200.rl.curriculum import Curriculum, CurriculumConfig, CurriculumTaskSource, evaluate_passk


def _cpython(program: str, args: tuple) -> str:
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        exec(compile(S.call_source(program, args), "<solve>", "exec"), {})  # package-written references only
    return buf.getvalue()


@pytest.mark.parametrize("fam", S.FAMILIES, ids=lambda f: f.key)
def test_reference_matches_cpython(fam):
    rng = random.Random(3)
    outs = set()
    for args in [fam.gen(rng) for _ in range(25)] + list(fam.edge):
        got = S.run_call(fam.reference, args, max_steps=10 * S.GRADE_STEPS)
        assert got.ok, (fam.key, args, got.error)
        assert got.stdout == _cpython(fam.reference, args), (fam.key, args)
        outs.add(got.stdout)
    assert len(outs) >= 2, fam.key


def test_levels_and_problem_makeup():
    assert sorted({f.level for f in S.FAMILIES}) == list(range(1, S.NUM_LEVELS + 1))
    assert all(len(S.families(lv)) == 3 for lv in range(1, S.NUM_LEVELS + 1))
    rng = random.Random(0)
    for lv in range(1, S.NUM_LEVELS + 1):
        p = S.sample_problem(rng, lv)
        fam = S.BY_KEY[p.family]
        assert p.level == lv and len(p.public_tests) == S.N_PUBLIC and len(p.hidden_tests) == S.N_HIDDEN
        assert len({repr(a) for a, _ in p.tests}) == len(p.tests)  # distinct calls
        hidden_args = [a for a, _ in p.hidden_tests]
        assert all(e in hidden_args for e in fam.edge[:S.N_HIDDEN])  # edge cases are graded
        assert fam.signature in p.prompt and "Examples:" in p.prompt
        for a, out in p.public_tests:
            assert out.strip() in p.prompt
    assert S.eval_problems(5, 4) == S.eval_problems(5, 4)


def test_grading_and_feedback():
    rng = random.Random(1)
    p = S.make_problem(S.BY_KEY["list_max"], rng)
    ref = S.BY_KEY["list_max"].reference
    g = S.grade(ref, p)
    assert g == {"has_code": 1.0, "ran_ok": 1.0, "frac_passed": 1.0, "exact": 1.0}
    assert S.reward_of(g) == pytest.approx(1.0) and S.feedback(ref, p) == ""
    assert S.SolveProblemEnv.reward(ref + "\nEND\ntrailing text", p) == pytest.approx(1.0)
    # no empty-list case: fails exactly the hidden edge test(s) with an error, so ran_ok drops
    naive = "def solve(xs):\n  m = xs[0]\n  for x in xs:\n    if x > m:\n      m = x\n  return m"
    gn = S.grade(naive, p)
    assert gn["ran_ok"] == 0.0 and 0.5 < gn["frac_passed"] < 1.0 and gn["exact"] == 0.0
    assert 0.4 < S.reward_of(gn) < 0.9
    const = "def solve(xs):\n  return 3"
    assert S.grade(const, p)["frac_passed"] < 0.5
    assert S.grade("print(1)", p)["has_code"] == 0.0 and S.reward_of(S.grade("print(1)", p)) == 0.0
    fb = S.feedback("def solve(xs):\n  return 0", p)
    assert fb.startswith("solve(") and "expected" in fb
    assert "raised" in S.feedback("def solve(xs):\n  return 1 / 0", p)
    assert S.feedback("x = 1", p) == "No function named solve was defined."


def test_curriculum_source_and_passk():
    env = S.SolveProblemEnv(seed=0)
    cur = Curriculum(CurriculumConfig(num_levels=S.NUM_LEVELS, steps_per_level=2, promote_threshold=0.5))
    src = CurriculumTaskSource(env, cur, seed=0)
    for _ in range(4):  # a policy that always writes the right function: levels unlock on schedule
        task = src.sample()
        prob = task.answer
        src.reward(S.BY_KEY[prob.family].reference + "\nEND", prob)
        src.on_step()
    assert cur.unlocked == 3
    probs = [q for lv in (1, 7) for q in env.held_out(lv, 3)]

    def policy(prob):
        return [S.BY_KEY[prob.family].reference, "def solve(*a):\n  return 0", "nonsense"]

    res = evaluate_passk(policy, probs, 1, solved=S.SolveProblemEnv.solved)
    assert res == {1: pytest.approx(1 / 3), 7: pytest.approx(1 / 3)}
    assert evaluate_passk(policy, probs, 3, solved=S.SolveProblemEnv.solved) == {1: 1.0, 7: 1.0}
