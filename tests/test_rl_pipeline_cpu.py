"""Segment SFT, greedy completion and the idempotent tuning-ladder runner on a tiny policy."""

import json
import os

import pytest
import torch

from marin_experiments_b200.data.tokenize import ByteTokenizer
from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
from marin_experiments_b200.rl import chat_sft, code_tasks, pipeline


def _tiny():
    cfg = Qwen3Config(vocab_size=257, hidden_dim=64, intermediate_dim=128, num_layers=1, num_heads=2, num_kv_heads=1,
                      head_dim=32, max_seq_len=1024)
    return Qwen3Model(cfg).init_weights(0)


def test_pack_segments_masks_only_trained_text():
    tok = ByteTokenizer()
    t, m = chat_sft.pack_segments([[("ab", 0), ("cd", 1)], [("x", 1)]], tok, 6)
    assert t.shape == (2, 6) and m[0].tolist() == [0, 0, 1, 1, 0, 0] and m[1].tolist() == [1, 0, 0, 0, 0, 0]
    assert tok.decode(t[0, :4].tolist()) == "abcd"


def test_segment_sft_memorises_a_program():
    torch.manual_seed(0)
    tok = ByteTokenizer()
    m = _tiny()
    task = code_tasks.eval_tasks()[0]
    segs = [code_tasks.sft_segments(task)]
    losses = chat_sft.run_segment_sft(m, tok, segs, chat_sft.ChatSFTConfig(steps=60, batch_size=1, lr=3e-3,
                                                                         max_seq_len=512))
    assert losses[-1] < 0.2 * losses[0]
    out = chat_sft.complete(m, tok, code_tasks.build_prompt(task.prompt), 40)
    assert code_tasks.extract_program(out) == task.solution


def test_ladder_runs_idempotently(tmp_path, monkeypatch):
    tiny = {"coding": [pipeline.Stage("fewshot", tiers=(0,)),
                       pipeline.Stage("sft", 4, sft_steps=2, tiers=(0,)),
                       pipeline.Stage("sft_grpo", 4, sft_steps=1, grpo_steps=1, group_size=2, prompts_per_step=1,
                                      tiers=(0,))],
            "multiturn": [pipeline.Stage("sft_grpo", 2, sft_steps=1, grpo_steps=1, group_size=2, prompts_per_step=1,
                                         kind="multiturn", tiers=(3,))],
            "tools": [pipeline.Stage("t1", 3, sft_steps=1, grpo_steps=1, group_size=2, prompts_per_step=1,
                                     kind="tools", depth=2)],
            "arithmetic": [pipeline.Stage("s2", 3, sft_steps=1, grpo_steps=1, group_size=2, prompts_per_step=1,
                                          kind="arith", depth=2)],
            "curriculum": [pipeline.Stage("sft_grpo", 3, sft_steps=1, grpo_steps=1, group_size=2,
                                          prompts_per_step=1, kind="solve", tiers=(1, 7))]}
    monkeypatch.setattr(pipeline, "EXPERIMENTS", tiny)
    tok = ByteTokenizer()
    built = []

    def make():
        built.append(1)
        return _tiny()

    d = str(tmp_path)
    assert [done for _, done in pipeline.plan("coding", d)] == [False, False, False]
    res = pipeline.run("coding", make, tok, d, max_program_tokens=8, seq_len=512)
    assert len(built) == 3 and set(res) == {"fewshot", "sft", "sft_grpo"}
    r = json.load(open(pipeline.results_path(d, "coding", "sft_grpo")))
    assert r["eval"]["total"] == len(code_tasks.FAMILIES[0]) and "grpo" in r and "sft" in r
    again = pipeline.run("coding", make, tok, d)  # everything is done: nothing is built or run
    assert len(built) == 3 and again["sft"]["eval"] == res["sft"]["eval"]
    os.remove(pipeline.results_path(d, "coding", "sft"))
    pipeline.run("coding", make, tok, d, max_program_tokens=8, seq_len=512)
    assert len(built) == 4
    mt = pipeline.run("multiturn", make, tok, d, max_program_tokens=8, seq_len=768, max_rounds=2)
    ev = mt["sft_grpo"]["eval"]
    assert set(ev) == {"first_solve", "best_solve", "mean_rounds"} and 1.0 <= ev["mean_rounds"] <= 2.0
    tl = pipeline.run("tools", make, tok, d, seq_len=512, eval_tools=3)["t1"]
    assert set(tl["eval"]) == {"tool/tool_call_rate", "tool/arg_acc", "arithmetic/solve_ratio"} and "grpo" in tl
    saved = pipeline.run("arithmetic", make, tok, d, seq_len=512, eval_tools=4, save_dir=str(tmp_path / "pol"))
    ar = saved["s2"]["eval"]
    from marin_experiments_b200.models.qwen3 import load_hf

    back = load_hf(saved["s2"]["checkpoint"], dtype=torch.float32)
    assert back.cfg.num_layers == 1 and os.path.exists(os.path.join(saved["s2"]["checkpoint"], "config.json"))
    assert set(ar) == {"arith/solve_ratio", "arith/solve_all", "arith/solve_none", "arith/format_rate"}
    cu = pipeline.run("curriculum", make, tok, d, seq_len=512, max_program_tokens=8)["sft_grpo"]
    assert set(cu["eval"]) == {"level1", "level7"} and "grpo" in cu
    assert pipeline.main(["--experiment", "coding", "--results-dir", d, "--dry-run"]) == 0


def test_tool_transcript_matches_environment():
    from marin_experiments_b200.rl import tools

    task = tools.chain_tasks(1, seed=4, depth=2)[0]
    segs = pipeline.tool_transcript(task)
    script = iter([t for t, m in segs if m])
    env = tools.rollout(lambda _: next(script), task)
    assert tools.total_reward(env) == pytest.approx(1.9)
    # the transcript is exactly what the environment renders for that episode
    assert "".join(t for t, _ in segs) == env.render()


def test_chat_stage_on_local_snapshot(tmp_path, monkeypatch):
    import json as _json

    from marin_experiments_b200.data import instruct
    from marin_experiments_b200.data.tokenize import ByteTokenizer

    root = tmp_path / "snap"
    d = root / "allenai/tulu-3-sft-mixture"
    d.mkdir(parents=True)
    with open(d / "train-0.jsonl", "w") as f:
        for i in range(80):
            f.write(_json.dumps({"messages": [{"role": "user", "content": f"say {i % 3}"},
                                             {"role": "assistant", "content": f"ok {i % 3}"}]}) + "\n")
    monkeypatch.setattr(instruct, "DEFAULT_MIX", {"allenai/tulu-3-sft-mixture": 1.0})
    monkeypatch.setattr(pipeline, "EXPERIMENTS", {"chat": [pipeline.Stage("sft", 40, sft_steps=30, kind="chat",
                                                                          lr_sft=3e-3)]})
    res = pipeline.run("chat", _tiny, ByteTokenizer(), str(tmp_path / "res"), seq_len=128, chat_root=str(root))["sft"]
    before, after = res["eval_before"]["heldout_assistant_loss"], res["eval"]["heldout_assistant_loss"]
    assert after < 0.7 * before
    segs = pipeline.chat_segments([{"role": "user", "content": "u"}, {"role": "assistant", "content": "a"}])
    assert [m for _, m in segs] == [0, 0, 0, 1] and segs[3][0] == "a<|im_end|>\n"
