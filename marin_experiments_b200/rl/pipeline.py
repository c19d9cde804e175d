"""Idempotent runner of the coding tuning ladders (tunix-delphi-rl/training/pipeline.py:72-311,
tunix-delphi-rl/training/train_coding.py:1-326, tunix-delphi-rl/training/train_multiturn.py:1-492).

Each round of tuning is a ``Stage`` declared as data: how many SFT transcripts to warm up on, how
many GRPO steps to take afterwards, and the kind of episode -- ``coding`` (write one program,
``rl.code_tasks``), ``multiturn`` (write, run, read the output, revise: ``rl.code_agent``) or
``tools`` (chained calculator calls of a given depth, ``rl.tools``; train_agentic.py of the same
project). Running a stage starts from a fresh policy (``make_model()``), warms it up with masked
SFT on transcripts in the RL prompt format (multi-turn transcripts include repair rounds, tool
transcripts their tool results as context), optionally runs GRPO (``rl.learner.GRPOLearner`` over
``CodeTaskEnv``, or ``rl.multiturn.MultiTurnGRPO`` over ``CodeAgentEnv`` / ``CalcToolEnv``),
evaluates greedily on held-out tasks and writes
``<results_dir>/<experiment>/<stage>.json``. A stage whose results file exists is skipped, so
re-running resumes the ladder; deleting one file re-runs that stage. ``plan`` (and ``--dry-run``)
lists which stages would run without building a model.

Four more kinds: ``chat`` (conversational SFT on the instruction / tool-use mixture of
``data.instruct`` read from local snapshots under ``MXK_SFT_SNAPSHOTS``, evaluated as the held-out
assistant-token loss before and after; launch_chat_sft.py), ``agent`` (terminal tasks in the sandbox, ``rl.terminal`` over the built-in
``rl.terminal_tasks``: SFT on oracle trajectories whose observations come from running them, then
multi-turn GRPO with the graded score as the episode reward, then the solve rate on held-out tasks;
the openthoughts-agent launchers), ``arith`` (staged few-shot arithmetic, ``rl.arithmetic``, stage = ``depth``;
train_delphi.py) and ``solve`` (the nine levels of test-graded ``def solve`` problems under the
curriculum, ``rl.solve_problems``; train_curriculum.py).

Ladders: ``coding`` -- few-shot only, SFT on 150 / 300 / 1000 transcripts, SFT 300 + GRPO;
``multiturn`` -- few-shot, SFT with repair rounds, SFT + multi-turn GRPO, on tiers 3-5; ``tools``
-- few-shot and SFT + GRPO at depths 1, 2 and 3 (stages T0-T2); ``arithmetic`` -- SFT + GRPO at
stages 0-3; ``curriculum`` -- few-shot, SFT, SFT + curriculum GRPO over levels 1-9; ``agent`` --
few-shot, SFT on 120 trajectories, SFT + GRPO; ``chat`` -- SFT on 2000 conversations.
"""

from __future__ import annotations

import json
import os
import random
import time
from collections.abc import Callable
from dataclasses import asdict, dataclass, field, replace

from . import code_agent, code_tasks
from .chat_sft import ChatSFTConfig, complete, run_segment_sft


@dataclass(frozen=True)
class Stage:
    name: str
    sft_examples: int = 0
    sft_steps: int = 0  # 0 -> 2 passes over the transcripts at the batch size
    grpo_steps: int = 0
    kind: str = "coding"  # coding | multiturn | tools | arith | solve | agent | chat
    depth: int = 1  # tools: calculator calls per task
    tiers: tuple[int, ...] = code_tasks.TIERS
    lr_sft: float = 3e-4
    lr_rl: float = 1e-5
    group_size: int = 8
    prompts_per_step: int = 4
    extra: dict = field(default_factory=dict)


_HARD = (3, 4, 5)
_ALL_LEVELS = tuple(range(1, 10))
EXPERIMENTS: dict[str, list[Stage]] = {
    "coding": [Stage("fewshot"), Stage("sft150", 150), Stage("sft300", 300), Stage("sft1000", 1000),
               Stage("sft300_grpo", 300, grpo_steps=60)],
    "multiturn": [Stage("fewshot", kind="multiturn", tiers=_HARD), Stage("sft300", 300, kind="multiturn", tiers=_HARD),
                  Stage("sft300_grpo", 300, grpo_steps=60, kind="multiturn", tiers=_HARD)],
    "tools": [Stage("fewshot", kind="tools"), Stage("t0", 200, grpo_steps=40, kind="tools", depth=1),
              Stage("t1", 200, grpo_steps=40, kind="tools", depth=2),
              Stage("t2", 200, grpo_steps=40, kind="tools", depth=3)],
    "arithmetic": [Stage(f"s{k}", 200, grpo_steps=40, kind="arith", depth=k) for k in range(4)],
    "curriculum": [Stage("fewshot", kind="solve", tiers=_ALL_LEVELS), Stage("sft300", 300, kind="solve", tiers=_ALL_LEVELS),
                   Stage("sft300_grpo", 300, grpo_steps=80, kind="solve", tiers=_ALL_LEVELS)],
    "chat": [Stage("sft2000", 2000, kind="chat")],
    "agent": [Stage("fewshot", kind="agent"), Stage("sft120", 120, kind="agent"),
              Stage("sft120_grpo", 120, grpo_steps=30, kind="agent", group_size=4)],
}


def results_path(results_dir: str, experiment: str, stage: str) -> str:
    return os.path.join(results_dir, experiment, f"{stage}.json")


def plan(experiment: str, results_dir: str, only: str | None = None) -> list[tuple[Stage, bool]]:
    """``[(stage, done)]`` for the ladder (or one stage of it)."""
    stages = EXPERIMENTS[experiment]
    if only is not None:
        stages = [s for s in stages if s.name == only]
        if not stages:
            raise KeyError(f"experiment {experiment!r} has no stage {only!r}")
    return [(s, os.path.exists(results_path(results_dir, experiment, s.name))) for s in stages]


def tool_transcript(task) -> list[tuple[str, int]]:
    """A solved chain in the tool environment's rendering: calls and the final answer trained."""
    from . import tools

    segs = [(f"{tools.SYSTEM_PROMPT}\n{task.prompt}\n", 0)]
    acc = task.operands[0]
    for v in task.operands[1:]:
        segs.append((f"CALC({acc} * {v})\n", 1))
        acc *= v
        segs.append((f"Tool result: {acc}\n", 0))
    segs.append((f"{acc}\n", 1))
    return segs


def agent_transcript(task, sandbox: str = "auto") -> list[tuple[str, int]]:
    """The oracle trajectory of a terminal task as ChatML segments: actions trained, the task and the
    terminal output (from actually running the actions) as context."""
    from ..data.chat import IM_END, IM_START, render_chatml
    from . import terminal, terminal_tasks

    env = terminal.TerminalEnv(max_turns=4, sandbox=sandbox)
    try:
        msgs = env.reset(task)
        segs = [(render_chatml(msgs[:1], add_generation_prompt=True), 0)]
        for act in terminal_tasks.oracle_actions(task):
            segs.append((act + IM_END, 1))
            obs, done = env.step(act)
            if done or obs is None:
                break
            segs.append((f"\n{IM_START}user\n{obs}{IM_END}\n{IM_START}assistant\n", 0))
        return segs
    finally:
        env.close()


def _agent_tasks(n: int, seed: int, root: str):
    from . import terminal, terminal_tasks

    d = os.path.join(root, f"seed{seed}-n{n}")
    if not os.path.isdir(d):
        terminal_tasks.write_tasks(d, n, seed)
    return terminal.load_tasks(d)


CHAT_HELDOUT = 32  # the first conversations of the stream are held out; training reads the ones after


def chat_segments(messages: list[dict]) -> list[tuple[str, int]]:
    """A conversation as ChatML segments: assistant contents with their end marker trained, the rest
    context (the masking of ``data.chat.encode_chat``)."""
    from ..data.chat import IM_END, IM_START

    segs = []
    for m in messages:
        segs.append((f"{IM_START}{m['role']}\n", 0))
        segs.append((f"{m['content']}{IM_END}\n", int(m["role"] == "assistant")))
    return segs


def _chat_rows(n: int, seed: int, root: str, skip: int = 0) -> list[list[dict]]:
    from ..data import instruct

    rows = list(instruct.chat_tooluse_mixture(root, seed=seed, limit=skip + n))
    return [r["messages"] for r in rows[skip:]]


def _transcripts(stage: Stage, seed: int, sandbox: str = "auto", task_root: str = "", chat_root: str = ""):
    rng = random.Random(seed)
    if stage.kind == "chat":
        return [chat_segments(m) for m in _chat_rows(stage.sft_examples, seed, chat_root, skip=CHAT_HELDOUT)]
    if stage.kind == "agent":
        return [agent_transcript(t, sandbox) for t in _agent_tasks(stage.sft_examples, seed, task_root)]
    if stage.kind == "arith":
        from . import arithmetic

        out = []
        for _ in range(stage.sft_examples):
            q, gold = arithmetic.make_problem(stage.depth, rng)
            out.append([(arithmetic.build_prompt(stage.depth, q), 0), (f" {gold}\n", 1)])
        return out
    if stage.kind == "solve":
        from . import solve_problems

        probs = [solve_problems.sample_problem(rng, rng.choice(stage.tiers)) for _ in range(stage.sft_examples)]
        return [[(p.prompt, 0), (solve_problems.BY_KEY[p.family].reference + "\nEND\n", 1)] for p in probs]
    if stage.kind == "tools":
        from . import tools

        return [tool_transcript(t) for t in tools.chain_tasks(stage.sft_examples, seed, stage.depth)]
    if stage.kind == "multiturn":
        rng = random.Random(seed + 1)
        tasks = code_agent.coding_tasks(stage.sft_examples, seed, stage.tiers)
        prefix = [(f"{code_agent.SYSTEM_PROMPT}\n", 0)]
        return [prefix + code_agent.sft_transcript(rng, t, fix_prob=0.3) for t in tasks]
    return [code_tasks.sft_segments(t) for t in code_tasks.sample_tasks(stage.sft_examples, seed, stage.tiers)]


def run_stage(stage: Stage, make_model: Callable, tok, *, seed: int = 0, eval_per_family: int = 1,
              max_program_tokens: int = 160, sft_batch: int = 8, seq_len: int = 1024, max_rounds: int = 3,
              eval_tools: int = 50, sandbox: str = "auto", task_root: str | None = None,
              agent_turns: int = 4, save_dir: str | None = None, chat_root: str | None = None) -> dict:
    """Run one stage from a fresh policy; with ``save_dir`` the trained policy is exported there as a
    Hugging Face Qwen3 checkpoint (safetensors + config.json), so a separate evaluation, RL or
    serving job can load it."""
    if stage.kind == "agent" and task_root is None:  # generated task directories live for this stage only
        import shutil
        import tempfile

        root = tempfile.mkdtemp(prefix="mxk-terminal-tasks-")
        try:
            return run_stage(stage, make_model, tok, seed=seed, eval_per_family=eval_per_family,
                             max_program_tokens=max_program_tokens, sft_batch=sft_batch, seq_len=seq_len,
                             max_rounds=max_rounds, eval_tools=eval_tools, sandbox=sandbox, task_root=root,
                             agent_turns=agent_turns, save_dir=save_dir, chat_root=chat_root)
        finally:
            shutil.rmtree(root, ignore_errors=True)
    model = make_model()
    t0 = time.time()
    out: dict = {"stage": asdict(stage), "seed": seed}
    chat_root = chat_root or os.environ.get("MXK_SFT_SNAPSHOTS", "")
    held_chat = None
    if stage.kind == "chat":  # held-out conversations: the assistant-token loss before and after SFT
        import torch

        from .chat_sft import masked_lm_loss, pack_segments

        held_chat = pack_segments([chat_segments(m) for m in _chat_rows(CHAT_HELDOUT, seed, chat_root)], tok, seq_len)

        def held_loss():
            dev = next(model.parameters()).device
            with torch.no_grad():
                return float(masked_lm_loss(model, held_chat[0].to(dev), held_chat[1].to(dev)))

        out["eval_before"] = {"heldout_assistant_loss": held_loss()}
    if stage.sft_examples:
        steps = stage.sft_steps or max(1, 2 * stage.sft_examples // sft_batch)
        cfg = ChatSFTConfig(steps=steps, batch_size=sft_batch, lr=stage.lr_sft, max_seq_len=seq_len, seed=seed)
        losses = run_segment_sft(model, tok, _transcripts(stage, seed, sandbox, task_root, chat_root), cfg)
        out["sft"] = {"steps": steps, "first_loss": losses[0], "last_loss": losses[-1]}
    if stage.kind not in ("coding", "multiturn", "tools", "arith", "solve", "agent", "chat"):
        raise ValueError(f"unknown stage kind {stage.kind!r}")
    if stage.grpo_steps:
        if stage.kind == "tools":
            from . import tools
            from .multiturn import MultiTurnConfig, MultiTurnGRPO

            chains = iter(tools.chain_tasks(stage.grpo_steps * stage.prompts_per_step, seed + 7, stage.depth))
            lr = MultiTurnGRPO(model, tok, lambda: next(chains), lambda t: tools.CalcToolEnv(t),
                               MultiTurnConfig(group_size=stage.group_size, lr=stage.lr_rl, stop="\n",
                                               max_turn_tokens=32, max_total_tokens=seq_len, seed=seed),
                               reward_fn=tools.total_reward)
        elif stage.kind == "multiturn":
            from .multiturn import MultiTurnConfig, MultiTurnGRPO

            tasks = iter(code_agent.coding_tasks(stage.grpo_steps * stage.prompts_per_step, seed + 7, stage.tiers))
            lr = MultiTurnGRPO(model, tok, lambda: next(tasks),
                               lambda t: code_agent.CodeAgentEnv(t, max_rounds=max_rounds),
                               MultiTurnConfig(group_size=stage.group_size, lr=stage.lr_rl, stop="\nEND\n",
                                               max_turn_tokens=max_program_tokens, max_total_tokens=seq_len,
                                               seed=seed))
        elif stage.kind == "agent":
            import itertools

            from ..data.chat import IM_END
            from .multiturn import MultiTurnConfig, MultiTurnGRPO
            from .terminal import ChatTerminalEnv

            pool = itertools.cycle(_agent_tasks(max(8, stage.prompts_per_step * 4), seed + 7, task_root))
            lr = MultiTurnGRPO(model, tok, lambda: next(pool), lambda t: ChatTerminalEnv(t, agent_turns, sandbox),
                               MultiTurnConfig(group_size=stage.group_size, lr=stage.lr_rl, stop=IM_END,
                                               max_turn_tokens=max_program_tokens, max_total_tokens=seq_len,
                                               seed=seed))
        elif stage.kind == "arith":
            from .arithmetic import ArithmeticEnv
            from .learner import GRPOConfig, GRPOLearner

            lr = GRPOLearner(model, tok, ArithmeticEnv(stage.depth, seed + 7),
                             GRPOConfig(group_size=stage.group_size, lr=stage.lr_rl, max_new_tokens=8, seed=seed))
        elif stage.kind == "solve":
            from .curriculum import Curriculum, CurriculumConfig, CurriculumTaskSource
            from .learner import GRPOConfig, GRPOLearner
            from .solve_problems import NUM_LEVELS, SolveProblemEnv

            cur = Curriculum(CurriculumConfig(num_levels=NUM_LEVELS, steps_per_level=max(1, stage.grpo_steps // 10)))
            lr = GRPOLearner(model, tok, CurriculumTaskSource(SolveProblemEnv(seed + 7), cur, seed),
                             GRPOConfig(group_size=stage.group_size, lr=stage.lr_rl,
                                        max_new_tokens=max_program_tokens, seed=seed))
        else:
            from .learner import GRPOConfig, GRPOLearner

            lr = GRPOLearner(model, tok, code_tasks.CodeTaskEnv(seed + 7, stage.tiers),
                             GRPOConfig(group_size=stage.group_size, lr=stage.lr_rl,
                                        max_new_tokens=max_program_tokens, seed=seed))
        hist = [lr.step(n_prompts=stage.prompts_per_step) for _ in range(stage.grpo_steps)]
        out["grpo"] = {"steps": len(hist), "reward_first": hist[0]["reward_mean"], "reward_last": hist[-1]["reward_mean"]}
    model.eval()
    ladder = [t for t in code_tasks.eval_tasks(eval_per_family) if t.tier in stage.tiers]
    if stage.kind == "chat":
        ev = {"heldout_assistant_loss": held_loss()}
    elif stage.kind == "agent":
        from ..data.chat import IM_END, render_chatml
        from . import terminal

        def model_fn(msgs):
            text = complete(model, tok, render_chatml(msgs, add_generation_prompt=True), max_program_tokens,
                            stops=(IM_END,))
            return text.split(IM_END, 1)[0]

        ev = terminal.evaluate(model_fn, _agent_tasks(eval_tools, 9_000_011, task_root), agent_turns, sandbox)
        ev.pop("episodes")
    elif stage.kind == "arith":
        from . import arithmetic

        erng = random.Random(3_000_017 + stage.depth)
        held = [arithmetic.make_problem(stage.depth, erng) for _ in range(eval_tools)]
        outs = [complete(model, tok, arithmetic.build_prompt(stage.depth, q), 8, stops=("\n",)) for q, _ in held]
        ev = arithmetic.group_metrics(outs, [g for _, g in held], 1)
        ev["arith/format_rate"] = sum(arithmetic.format_reward(o) > 0 for o in outs) / max(len(outs), 1)
    elif stage.kind == "solve":
        from . import solve_problems

        ev = {}
        for lv in stage.tiers:
            probs = solve_problems.eval_problems(lv, 3 * eval_per_family)
            ok = [solve_problems.SolveProblemEnv.solved(complete(model, tok, p.prompt, max_program_tokens), p)
                  for p in probs]
            ev[f"level{lv}"] = sum(ok) / len(ok)
    elif stage.kind == "tools":
        from . import tools

        held = tools.chain_tasks(eval_tools, 1_000_003 + stage.depth, stage.depth)
        envs = [tools.rollout(lambda text: complete(model, tok, text, 32, stops=("\n",)), t) for t in held]
        ev = tools.metrics(envs, [tools.total_reward(e) for e in envs])
    elif stage.kind == "multiturn":
        tasks = [code_agent.CodingTask(t.prompt, t.solution, t.gold) for t in ladder]
        ev = code_agent.evaluate_multiturn(lambda text: complete(model, tok, text, max_program_tokens),
                                           tasks, max_rounds=max_rounds)
        ev.pop("envs")
    else:
        ev = code_tasks.evaluate(lambda p: complete(model, tok, p, max_program_tokens), ladder)
    out["eval"] = ev
    if save_dir:
        from ..models.qwen3_export import export_hf

        out["checkpoint"] = export_hf(model, os.path.join(save_dir, stage.name))
    out["seconds"] = time.time() - t0
    return out


def run(experiment: str, make_model: Callable, tok, results_dir: str, *, only: str | None = None,
        overrides: dict | None = None, **kw) -> dict[str, dict]:
    """Run the stages of ``experiment`` that have no results yet; returns every stage's results."""
    res = {}
    for stage, done in plan(experiment, results_dir, only):
        path = results_path(results_dir, experiment, stage.name)
        if done:
            with open(path) as f:
                res[stage.name] = json.load(f)
            continue
        st = replace(stage, **(overrides or {}))
        r = run_stage(st, make_model, tok, **kw)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        tmp = path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(r, f, indent=1)
        os.replace(tmp, path)
        res[stage.name] = r
    return res


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(prog="python -m marin_experiments_b200.rl.pipeline")
    ap.add_argument("--experiment", choices=sorted(EXPERIMENTS), default="coding")
    ap.add_argument("--stage", default=None)
    ap.add_argument("--results-dir", default="rl_results")
    ap.add_argument("--model-dir", default=os.environ.get("MXK_POLICY_DIR", ""),
                    help="Hugging Face Qwen3 checkpoint directory (safetensors + tokenizer.json)")
    ap.add_argument("--model", default=os.environ.get("MXK_POLICY", ""),
                    help="registered base model (models.registry): the checkpoint is checked against it")
    ap.add_argument("--save-policies", default="", help="export each stage's trained policy under this directory")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    for stage, done in plan(a.experiment, a.results_dir, a.stage):
        print(f"[{'done' if done else 'todo'}] {a.experiment}/{stage.name}: sft={stage.sft_examples} "
              f"grpo={stage.grpo_steps} kind={stage.kind} tiers={list(stage.tiers)} depth={stage.depth}")
    if a.dry_run:
        return 0
    if not a.model_dir:
        raise SystemExit("--model-dir (or MXK_POLICY_DIR) is required to run stages")
    import torch

    from ..data.tokenize import load_tokenizer
    from ..models import registry
    from ..models.qwen3 import load_hf

    tok = load_tokenizer(a.model_dir)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if a.model:
        registry.check_checkpoint(a.model, a.model_dir)
    res = run(a.experiment, lambda: load_hf(a.model_dir, device=dev, dtype=torch.float32), tok, a.results_dir,
              only=a.stage, save_dir=(os.path.join(a.save_policies, a.experiment) if a.save_policies else None))
    import shutil

    for name, r in res.items():
        ck = r.get("checkpoint")
        if ck and os.path.isdir(ck):  # the exported policy loads with its tokenizer
            for fn in ("tokenizer.json", "tokenizer_config.json"):
                if os.path.exists(os.path.join(a.model_dir, fn)):
                    shutil.copy(os.path.join(a.model_dir, fn), os.path.join(ck, fn))
        print(name, json.dumps(r["eval"]))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
