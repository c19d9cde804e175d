"""Tiered coding-task families (checked against CPython), the eval ladder, and staged arithmetic."""

import contextlib
import io
import random

import pytest

from marin_experiments_b200.rl import arithmetic as ar
from marin_experiments_b200.rl import code_tasks as ct


def _cpython(src: str) -> str:
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        exec(compile(src, "<task>", "exec"), {})  # reference solutions written in this package only
    return buf.getvalue()


@pytest.mark.parametrize("tier", ct.TIERS)
def test_families_match_cpython_and_vary(tier):
    for fam in ct.FAMILIES[tier]:
        rng = random.Random(7)
        golds = set()
        for _ in range(25):
            t = ct.make_task(rng, tier, fam)
            assert t.gold == _cpython(t.solution), (fam.__name__, t.solution)
            golds.add(t.gold)
        assert len(golds) >= 2, fam.__name__  # the gold changes with the parameters


def test_prompt_extract_and_reward():
    rng = random.Random(0)
    t = ct.make_task(rng, 4)
    p = ct.build_prompt(t.prompt)
    assert p.startswith(ct.CODE_FEWSHOT) and p.endswith(f"Task: {t.prompt}\n")
    assert ct.extract_program("print(1)\nEND\nprint(2)") == "print(1)"
    assert ct.extract_program("print(1)\nTask: next") == "print(1)"
    assert ct.extract_program("END") == "" and ct.extract_program("") == ""
    assert ct.code_reward(t.solution + "\nEND\ngarbage", t.gold) == 2.0
    wrong = ct.code_reward("print('x')\nEND", t.gold)
    assert 0.4 <= wrong < 1.0
    assert ct.code_reward("print(1/0)\nEND", t.gold) == pytest.approx(0.1)
    assert ct.code_reward("END", t.gold) == 0.0
    m = ct.code_metrics([t.solution, "print(1/0)", ""], [t.gold] * 3)
    assert m == {"code/has_code": 2 / 3, "code/ran_ok": 1 / 3, "code/solve_ratio": 1 / 3}


def test_eval_ladder_and_harness():
    ev = ct.eval_tasks()
    assert ev == ct.eval_tasks() and len(ev) == sum(len(v) for v in ct.FAMILIES.values())
    assert {t.family for t in ev} == {f.__name__.lstrip("_") for v in ct.FAMILIES.values() for f in v}
    by_prompt = {ct.build_prompt(t.prompt): t for t in ev}
    res = ct.evaluate(lambda p: by_prompt[p].solution + "\nEND\n", ev)
    assert res["solved"] == res["total"] == len(ev) and all(res[f"tier{k}"] == 1.0 for k in ct.TIERS)
    res0 = ct.evaluate(lambda p: "print(0)\nEND\n", ev)
    assert res0["solved"] < len(ev) // 4
    env = ct.CodeTaskEnv(seed=3, tiers=(3,))
    task = env.sample()
    assert task.prompt.startswith(ct.CODE_FEWSHOT) and env.reward("print(0)\nEND", task.answer) < 1.0
    seg = ct.sft_segments(ev[0])
    assert [m for _, m in seg] == [0, 1] and seg[1][0].endswith("\nEND\n")


def test_arithmetic_stages():
    rng = random.Random(1)
    for stage in ar.STAGES:
        for _ in range(200):
            q, gold = ar.make_problem(stage, rng)
            if stage < 3:
                expr = q[len("Q: "):q.index(" =")]
                assert eval(expr) == int(gold)  # noqa: S307 -- expressions built above from integers
                if stage == 1 and "-" in expr:
                    assert int(gold) >= 0
            else:
                lhs, c = q[len("Solve for x: "):].split(" = ")
                c = int(c.split(";")[0])
                x = int(gold)
                assert eval(lhs.replace("x", f"({x})").replace("*", "*")) == c  # noqa: S307
            p = ar.build_prompt(stage, q)
            assert p.startswith(ar.FEWSHOT[stage]) and (p.endswith("A:") or p.endswith("x ="))
    assert ar.parse_answer(" 42\nQ: 1 + 1 =") == 42 and ar.parse_answer(" -7") == -7
    assert ar.parse_answer(" the answer is 12") == 12 and ar.parse_answer(" none") is None
    assert ar.total_reward(" 17\n", "17") == pytest.approx(1.1)
    assert ar.total_reward(" 18\n", "17") == pytest.approx(0.1 + 0.5 / (1 + 1 / 1.7))
    assert ar.total_reward(" 18\n", "17", dense=False) == pytest.approx(0.1)
    assert ar.total_reward(" nothing", "17") == 0.0
    m = ar.group_metrics([" 1", " 1", " 2", " 3"], ["1", "1", "1", "1"], 2)
    assert m == {"arith/solve_ratio": 0.5, "arith/solve_all": 0.5, "arith/solve_none": 0.5}
    env = ar.ArithmeticEnv(stage=2, seed=0)
    t = env.sample()
    assert env.reward(f" {t.answer}", t.answer) > 1.0
