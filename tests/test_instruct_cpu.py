"""Instruction datasets: row layouts to chat messages, local snapshots, the weighted interleave and
the chat token cache."""

import gzip
import json
import os

import pytest

from marin_experiments_b200.data import instruct as I


def test_layouts():
    tulu = I.DATASETS["allenai/tulu-3-sft-mixture"]
    row = {"messages": [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"},
                        {"role": "assistant", "content": "<think>x</think>hello"}], "dataset": "d", "id": 3}
    out = I.transform_row(row, tulu)
    assert [m["role"] for m in out["messages"]] == ["system", "user", "assistant"]
    assert out["messages"][2]["content"] == "<|start_think|>x<|end_think|>hello"
    assert out["metadata"] == {"dataset": "d", "id": 3, "source": ""}
    assert I.transform_row({"messages": [{"role": "narrator", "content": "?"}]}, tulu) is None
    assert I.transform_row({"messages": []}, tulu) is None

    oh = I.transform_row({"conversations": [{"from": "human", "value": "q"}, {"from": "gpt", "value": "a"}],
                          "id": "1", "category": "c", "source": "s"}, I.DATASETS["teknium/OpenHermes-2.5"])
    assert oh["messages"] == [{"role": "user", "content": "q"}, {"role": "assistant", "content": "a"}]

    mm = I.transform_row({"query": "2+2?", "response": "4", "type": "GSM"}, I.DATASETS["meta-math/MetaMathQA"])
    assert mm["messages"][1] == {"role": "assistant", "content": "4"} and mm["metadata"] == {"type": "GSM"}
    assert I.transform_row({"query": None, "response": "4"}, I.DATASETS["meta-math/MetaMathQA"]) is None

    nr = I.transform_row({"question": "why", "responses": [{"response": "because"}], "reference_answer": "r"},
                         I.DATASETS["facebook/natural_reasoning"])
    assert nr["messages"][1]["content"] == "because"

    best = I.DatasetSpec("x/y", "0", I.Adapter("instruction_response", prompt_column="p", response_column="r",
                                                  best_of="pass_rate", content_key="code"))
    got = I.transform_row({"p": "sort", "r": [{"code": "a", "pass_rate": 0.2}, {"code": "b", "pass_rate": 0.9}]}, best)
    assert got["messages"][1]["content"] == "b"

    ml = I.DatasetSpec("x/z", "0", I.Adapter("message_list_response", prompt_column="p", response_column="r"))
    assert I.transform_row({"p": [{"role": "user", "content": "q"}], "r": "a"}, ml)["messages"][0]["content"] == "q"
    assert I.transform_row({"p": [{"role": "user", "content": "q"}] * 2, "r": "a"}, ml) is None
    assert I.transform_row({"p": [{"content": "q"}], "r": "a"}, ml) is None
    with pytest.raises(ValueError):
        I.Adapter("csv")
    assert set(I.DEFAULT_MIX) == {I.TULU[0], *I.TOOLUSE} and abs(sum(I.DEFAULT_MIX.values()) - 1.0) < 1e-9


def _snapshot(root, spec, rows, kind, split=""):
    d = os.path.join(root, spec.hf_id, spec.subset, split)
    os.makedirs(d, exist_ok=True)
    if kind == "parquet":
        import pyarrow as pa
        import pyarrow.parquet as pq

        pq.write_table(pa.Table.from_pylist(rows), os.path.join(d, "part-0.parquet"))
    else:
        with gzip.open(os.path.join(d, "part-0.jsonl.gz"), "wt") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")


def test_snapshots_mixture_and_cache(tmp_path):
    root = str(tmp_path / "snap")
    chat = [{"messages": [{"role": "user", "content": f"q{i}"}, {"role": "assistant", "content": f"a{i}"}],
             "dataset": "t", "id": i, "source": "s"} for i in range(300)]
    _snapshot(root, I.DATASETS["allenai/tulu-3-sft-mixture"], chat, "parquet")
    for k, name in enumerate(I.TOOLUSE):
        spec = I.DATASETS[name]
        rows = [{"messages": [{"role": "user", "content": f"t{k}-{i}"}, {"role": "assistant", "content": "call"},
                              {"role": "tool", "content": "42"}, {"role": "assistant", "content": "42"}]}
                for i in range(40)]
        _snapshot(root, spec, rows, "jsonl", spec.splits[0])
        # another split of the same repository must not leak into this one
        _snapshot(root, spec, [{"messages": [{"role": "user", "content": "other"}]}], "jsonl", "other_split")
    got = list(I.load_messages("smoltalk2-xlam", root))
    assert len(got) == 40 and all(r["messages"][0]["content"].startswith("t0-") for r in got)
    assert [m["role"] for m in got[0]["messages"]] == ["user", "assistant", "tool", "assistant"]

    mix = list(I.chat_tooluse_mixture(root, seed=1, limit=200))
    counts = I.source_counts(mix)
    assert len(mix) == 200 and 140 <= counts[I.TULU[0]] <= 195
    assert mix == list(I.chat_tooluse_mixture(root, seed=1, limit=200))  # deterministic
    everything = list(I.chat_tooluse_mixture(root, seed=2))  # exhausted sources drop out
    assert len(everything) == 300 + 3 * 40
    with pytest.raises(FileNotFoundError, match="no local snapshot"):
        list(I.load_messages("meta-math/MetaMathQA", root))

    from marin_experiments_b200.data.chat import write_chat_cache
    from marin_experiments_b200.data.tokenize import ByteTokenizer

    path = str(tmp_path / "mix.jsonl")
    assert I.write_messages_jsonl(mix[:50], path) == 50
    meta = write_chat_cache([path], str(tmp_path / "cache"), ByteTokenizer())
    assert meta["num_docs"] == 50 and meta["format"] == "chat"


def test_more_registry_entries_and_multi_subset(tmp_path):
    root = str(tmp_path / "snap")
    spec = I.DATASETS["cognitivecomputations/dolphin-r1-reasoning"]
    for sub, n in (("reasoning-deepseek", 3), ("reasoning-flash", 2)):
        _snapshot(root, I.DatasetSpec(spec.hf_id, spec.revision, spec.adapter, spec.metadata_columns, sub),
                  [{"messages": [{"role": "user", "content": f"{sub}-{i}"}], "answer": "a", "score": 5}
                   for i in range(n)], "jsonl")
    got = list(I.load_messages("cognitivecomputations/dolphin-r1-reasoning", root))
    assert [r["messages"][0]["content"] for r in got] == ["reasoning-deepseek-0", "reasoning-deepseek-1",
                                                          "reasoning-deepseek-2", "reasoning-flash-0",
                                                          "reasoning-flash-1"]
    assert got[0]["metadata"]["score"] == 5
    omr = I.DATASETS["nvidia/OpenMathReasoning/tir"]
    _snapshot(root, omr, [{"problem": "p", "generated_solution": "tir"}], "jsonl", "tir")
    _snapshot(root, omr, [{"problem": "p", "generated_solution": "cot"}], "jsonl", "cot")
    assert [r["messages"][1]["content"] for r in I.load_messages("nvidia/OpenMathReasoning/tir", root)] == ["tir"]
    ace = I.transform_row({"question": "q", "inferences": [{"completion": "x", "pass_rate": 0.1},
                                                           {"completion": "y", "pass_rate": 1.0}], "id": 1},
                          I.DATASETS["TIGER-Lab/AceCode-89K"])
    assert ace["messages"][1]["content"] == "y"
    bs = I.transform_row({"conversations": [{"from": "user", "value": "u"}, {"from": "assistant", "value": "v"}]},
                         I.DATASETS["bespokelabs/Bespoke-Stratos-17k"])
    assert [m["role"] for m in bs["messages"]] == ["user", "assistant"]
    assert len(I.DATASETS) >= 25
