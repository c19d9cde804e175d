"""Built-in terminal tasks in the task-directory format of ``rl.terminal``: small file and text
chores with a grader script and an oracle solution each, generated with random contents so an
answer cannot be memorised. They let the agent ladder (SFT on oracle trajectories, GRPO in the
sandbox, evaluation) run end to end without an external task set (openthoughts-agent/eval/tb_tasks.py
loads Terminal-Bench tasks of the same layout from a dataset).

Families: count the lines of a file; the largest number in a file; the lines of a file sorted; a
word replaced throughout a file; a directory with a file of given content; the number of files with
an extension. Each writes ``answer.txt`` (or the named output) in the working directory; its
``tests/test.sh`` writes ``1`` or ``0`` to ``reward.txt``.
"""

from __future__ import annotations

import json
import os
import random

_WORDS = ("alpha", "bravo", "delta", "echo", "gamma", "kilo", "lima", "oscar", "sierra", "tango")


def _write(path: str, text: str, mode: int | None = None) -> None:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w") as f:
        f.write(text)
    if mode is not None:
        os.chmod(path, mode)


def _family(rng: random.Random, k: int) -> tuple[str, dict[str, str], str, str]:
    """(instruction, starting files, grader body, oracle shell commands)."""
    if k == 0:
        lines = [rng.choice(_WORDS) for _ in range(rng.randint(3, 30))]
        return ("Write the number of lines in data.txt to answer.txt.", {"data.txt": "\n".join(lines) + "\n"},
                f'[ "$(tr -d " \\n" < answer.txt)" = "{len(lines)}" ]', "wc -l < data.txt > answer.txt\n")
    if k == 1:
        nums = [rng.randint(-500, 5000) for _ in range(rng.randint(4, 20))]
        return ("numbers.txt holds one integer per line. Write the largest of them to answer.txt.",
                {"numbers.txt": "\n".join(map(str, nums)) + "\n"},
                f'[ "$(tr -d " \\n" < answer.txt)" = "{max(nums)}" ]', "sort -n numbers.txt | tail -1 > answer.txt\n")
    if k == 2:
        lines = rng.sample(_WORDS, rng.randint(3, len(_WORDS)))
        want = "\n".join(sorted(lines)) + "\n"
        return ("Write the lines of names.txt in alphabetical order to sorted.txt.",
                {"names.txt": "\n".join(lines) + "\n", "tests/want.txt": want},
                "cmp -s sorted.txt tests/want.txt", "LC_ALL=C sort names.txt > sorted.txt\n")
    if k == 3:
        old, new = rng.sample(_WORDS, 2)
        text = " ".join(rng.choice(_WORDS[:4] + (old,)) for _ in range(rng.randint(8, 20))) + f" {old}\n"
        return (f"Replace every occurrence of the word {old} in story.txt with {new}, editing the file in place.",
                {"story.txt": text, "tests/want.txt": text.replace(old, new)},
                "cmp -s story.txt tests/want.txt", f"sed -i 's/{old}/{new}/g' story.txt\n")
    if k == 4:
        d, w = rng.choice(_WORDS), rng.choice(_WORDS)
        return (f"Create a directory named {d} containing a file note.txt whose only line is {w}.", {},
                f'[ -d {d} ] && [ "$(cat {d}/note.txt)" = "{w}" ]', f"mkdir -p {d} && echo {w} > {d}/note.txt\n")
    ext = rng.choice(["log", "csv", "md"])
    names = {f"files/{rng.choice(_WORDS)}{i}.{rng.choice(['log', 'csv', 'md', 'txt'])}": "x\n" for i in range(8)}
    count = sum(n.endswith("." + ext) for n in names)
    return (f"Write to answer.txt how many files in the directory files end in .{ext}.", names,
            f'[ "$(tr -d " \\n" < answer.txt)" = "{count}" ]', f"ls files | grep -c '\\.{ext}$' > answer.txt\n")


FAMILIES = 6


def write_task(root: str, task_id: str, rng: random.Random, family: int | None = None) -> str:
    k = rng.randrange(FAMILIES) if family is None else family
    instruction, files, check, solve = _family(rng, k)
    d = os.path.join(root, task_id)
    _write(os.path.join(d, "instruction.md"), instruction + "\n")
    _write(os.path.join(d, "task.toml"), "[agent]\ntimeout_sec = 60\n[verifier]\ntimeout_sec = 20\n")
    tests = {n: t for n, t in files.items() if n.startswith("tests/")}
    for name, text in files.items():
        if not name.startswith("tests/"):
            _write(os.path.join(d, "environment", name), text)
    for name, text in tests.items():
        _write(os.path.join(d, name), text)
    _write(os.path.join(d, "tests", "test.sh"),
           f"if {check}; then echo 1 > reward.txt; else echo 0 > reward.txt; fi\n", 0o755)
    _write(os.path.join(d, "solution", "solve.sh"), solve, 0o755)
    return d


def write_tasks(root: str, n: int, seed: int = 0) -> list[str]:
    rng = random.Random(seed)
    return [write_task(root, f"task-{seed}-{i:04d}", rng, i % FAMILIES) for i in range(n)]


def oracle_actions(task) -> list[str]:
    """The oracle trajectory as JSON actions: run the solution's commands, then declare the task done."""
    with open(os.path.join(task.root, "solution", "solve.sh")) as f:
        cmds = f.read()
    run = {"analysis": "The task is described above.", "plan": "Run the commands that produce the output.",
           "commands": [{"keystrokes": cmds, "duration": 1.0}], "task_complete": False}
    done = {"analysis": "The output is written.", "plan": "Finish.", "commands": [], "task_complete": True}
    return [json.dumps(run), json.dumps(done)]
