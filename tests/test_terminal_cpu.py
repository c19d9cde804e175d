"""Terminal tasks: JSON actions, the agent loop in the sandbox, test-script grading, the reset /
step environment and agent traces."""

import json
import os

from marin_experiments_b200.rl import terminal as T


def _task(root, tid="count-lines", with_reward_file=True):
    d = os.path.join(root, tid)
    os.makedirs(os.path.join(d, "environment"))
    os.makedirs(os.path.join(d, "tests"))
    os.makedirs(os.path.join(d, "solution"))
    open(os.path.join(d, "instruction.md"), "w").write("Write the number of lines of data.txt to answer.txt.\n")
    open(os.path.join(d, "task.toml"), "w").write("[agent]\ntimeout_sec = 120\n[verifier]\ntimeout_sec = 20\n")
    open(os.path.join(d, "environment", "data.txt"), "w").write("a\nb\nc\n")
    open(os.path.join(d, "environment", "Dockerfile"), "w").write("FROM scratch\n")
    if with_reward_file:
        test = ("mkdir -p logs/verifier\n"
                "if [ \"$(cat answer.txt 2>/dev/null | tr -d ' \\n')\" = 3 ]; then echo 1 > logs/verifier/reward.txt;"
                " else echo 0 > logs/verifier/reward.txt; fi\n")
    else:
        test = "test \"$(cat answer.txt 2>/dev/null | tr -d ' \\n')\" = 3\n"
    open(os.path.join(d, "tests", "test.sh"), "w").write(test)
    open(os.path.join(d, "solution", "solve.sh"), "w").write("wc -l < data.txt > answer.txt\n")
    return d


def _act(keys, done=False, prose=True):
    obj = {"analysis": "look {at} this \"quoted\"", "plan": "p",
           "commands": [{"keystrokes": k, "duration": 0.1} for k in keys], "task_complete": done}
    s = json.dumps(obj)
    return ("Sure, here is my action: " + s + " hope that helps {") if prose else s


def test_parse_action():
    a = T.parse_action(_act(["ls\n"]))
    assert a.ok and a.commands[0]["keystrokes"] == "ls\n" and not a.task_complete
    assert T.parse_action('{"plan": "x"} {"commands": []}').ok  # last object with commands
    assert not T.parse_action("no json here").ok and not T.parse_action('{"commands": "ls"}').ok
    assert T.parse_action('{"commands": [{"keystrokes": 3}, {"keystrokes": "pwd\\n"}]}').commands == \
        [{"keystrokes": "pwd\n"}]
    assert T.format_observation("x" * 20, limit=5).endswith("xxxxx") and "15 characters cut" in \
        T.format_observation("x" * 20, limit=5)


def test_episode_solves_and_grades(tmp_path):
    root = str(tmp_path / "tasks")
    _task(root)
    _task(root, "exit-code", with_reward_file=False)
    tasks = T.load_tasks(root)
    assert [t.task_id for t in tasks] == ["count-lines", "exit-code"]
    assert tasks[0].agent_timeout_s == 120 and tasks[0].verifier_timeout_s == 20

    def solver(msgs):
        # first turn: inspect; then solve; then declare done
        n = sum(m["role"] == "assistant" for m in msgs)
        if n == 0:
            return _act(["ls\n", "cat data.txt\n"])
        if n == 1:
            assert "data.txt" in msgs[-1]["content"] and "Dockerfile" not in msgs[-1]["content"]
            return "not json at all"
        if n == 2:
            assert msgs[-1]["content"] == T.PARSE_FAIL
            return _act(["wc -l < data.txt > answer.txt\n"])
        return _act([], done=True, prose=False)

    res = T.evaluate(solver, tasks, max_turns=8, sandbox="local")
    assert res["solved"] == 2 and res["mean_score"] == 1.0 and res["parse_failures"] == 2
    ep = res["episodes"][0]
    assert ep.turns == 4 and [m["role"] for m in ep.messages][:3] == ["user", "assistant", "user"]

    wrong = T.evaluate(lambda msgs: _act(["echo 7 > answer.txt\n"], done=False), tasks[:1], max_turns=2,
                       sandbox="local")
    assert wrong["solved"] == 0 and wrong["mean_score"] == 0.0 and wrong["mean_turns"] == 2


def test_env_reset_step_and_traces(tmp_path):
    root = str(tmp_path / "tasks")
    task = T.load_task(_task(root))
    env = T.TerminalEnv(max_turns=3, sandbox="local")
    try:
        msgs = env.reset(task)
        assert msgs[0]["role"] == "user" and task.instruction in msgs[0]["content"]
        obs, done = env.step(_act(["wc -l < data.txt > answer.txt\n", "cat answer.txt\n"]))
        assert not done and "3" in obs
        obs, done = env.step(_act([], done=True))
        assert done and obs is None and env.final_reward() == 1.0
    finally:
        env.close()

    import pyarrow as pa
    import pyarrow.parquet as pq

    rows = [{"conversations": [{"role": "user", "content": "task"}, {"role": "assistant", "content": _act(["ls\n"])}],
             "agent": "terminus", "model": "m", "task": "t", "episode": "0", "run_id": "r", "trial_name": "x"}]
    p = str(tmp_path / "traces.parquet")
    pq.write_table(pa.Table.from_pylist(rows), p)
    got = list(T.load_agent_traces(p))
    assert got[0]["messages"][1]["role"] == "assistant" and got[0]["metadata"]["agent"] == "terminus"
    assert T.parse_action(got[0]["messages"][1]["content"]).ok


def test_agent_cannot_write_its_own_score(tmp_path):
    """A task graded by exit status: a reward file the agent writes is removed before grading."""
    root = str(tmp_path / "tasks")
    task = T.load_task(_task(root, "exit-only", with_reward_file=False))
    cheat = _act(["echo 1 > reward.txt\n", "mkdir -p logs/verifier && echo 1 > logs/verifier/reward.txt\n",
                  "mkdir -p tests && ln -s ../outside.txt tests/test.sh\n"])
    res = T.evaluate(lambda msgs: cheat if len(msgs) == 1 else _act([], done=True), [task], max_turns=3,
                     sandbox="local")
    assert res["solved"] == 0 and res["mean_score"] == 0.0
    assert not (tmp_path / "outside.txt").exists()
