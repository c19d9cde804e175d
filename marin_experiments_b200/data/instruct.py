"""Instruction / chat SFT datasets: rows of several source layouts normalised to chat messages, a
registry of the datasets used for chat and tool-use SFT, and a weighted interleave of them
(tunix-delphi-rl/sft_data/instruction_datasets.py:80-682).

Every source row becomes ``{"messages": [{"role", "content"}, ...], "metadata": {...}}`` with roles
in ``system / user / assistant / tool``, or ``None`` when the row cannot be turned into a
conversation (it is skipped, never emitted empty). Source layouts (``Adapter.layout``):

* ``messages`` -- one column holds the conversation as a list of dicts; the role and content key
  names and the role values are configurable (``from`` / ``value`` with ``human`` / ``gpt`` for
  OpenHermes). A message whose role is not one of the four is a row error: the row is skipped.
* ``instruction_response`` -- a prompt column and a response column give one user and one assistant
  turn; with ``best_of`` the response column is a list of dicts and the one with the largest
  ``best_of`` value supplies ``content_key``.
* ``instruction_list_response`` -- the response column is a list whose first dict supplies
  ``content_key``.
* ``message_list_response`` -- the prompt column is a one-message list (rows with more messages,
  or whose message lacks the role key, are skipped) and the response column a string.

String contents get text replacements (by default the reasoning tags ``<think>`` / ``</think>``
become ``<|start_think|>`` / ``<|end_think|>``) and the spec's metadata columns are copied.

The machine that trains has no network, so rows are read from a local snapshot of each dataset:
``<root>/<hf id>/`` holding Parquet, JSON-lines (optionally gzipped) or JSON files, optionally
under per-split directories (``iter_rows``). ``interleave`` draws the next row from a source chosen
by weight, drops exhausted sources (the others' weights renormalise) and stops at ``limit``;
``chat_tooluse_mixture`` is the default blend, about 85 % general chat and 15 % tool use split
evenly across three tool-calling sets. ``write_messages_jsonl`` writes rows for
``data.chat.write_chat_cache``.
"""

from __future__ import annotations

import glob
import gzip
import json
import os
import random
from collections.abc import Callable, Iterable, Iterator
from dataclasses import dataclass

ROLES = ("system", "user", "assistant", "tool")
THINK_TAGS = {"<think>": "<|start_think|>", "</think>": "<|end_think|>"}
LAYOUTS = ("messages", "instruction_response", "instruction_list_response", "message_list_response")


@dataclass(frozen=True)
class Adapter:
    layout: str = "messages"
    conversation_column: str = "messages"
    prompt_column: str = ""
    response_column: str = ""
    role_key: str = "role"
    content_key: str = "content"
    role_values: tuple[tuple[str, str], ...] = ()  # (source value, chat role) besides the identity
    best_of: str = ""
    replacements: tuple[tuple[str, str], ...] | None = None  # None -> THINK_TAGS
    extra_metadata: Callable[[dict], dict] | None = None

    def __post_init__(self):
        if self.layout not in LAYOUTS:
            raise ValueError(f"unknown layout {self.layout!r}; one of {LAYOUTS}")

    def _role(self, value) -> str | None:
        mapped = dict(self.role_values).get(value, value)
        return mapped if mapped in ROLES else None

    def to_messages(self, row: dict) -> list[dict] | None:
        if self.layout == "messages":
            conv = row.get(self.conversation_column)
            if not conv:
                return None
            out = []
            for m in conv:
                role = self._role(m.get(self.role_key)) if isinstance(m, dict) else None
                if role is None or m.get(self.content_key) is None:
                    return None
                out.append({"role": role, "content": m[self.content_key]})
            return out
        prompt, resp = row.get(self.prompt_column), row.get(self.response_column)
        if prompt is None or resp is None:
            return None
        if self.layout == "instruction_response":
            if self.best_of:
                cands = [c for c in resp if isinstance(c, dict) and c.get(self.best_of) is not None]
                if not cands:
                    return None
                resp = max(cands, key=lambda c: c[self.best_of])[self.content_key]
        elif self.layout == "instruction_list_response":
            if not resp or not isinstance(resp[0], dict) or self.content_key not in resp[0]:
                return None
            resp = resp[0][self.content_key]
        else:  # message_list_response
            if len(prompt) != 1 or not isinstance(prompt[0], dict) or self.role_key not in prompt[0]:
                return None
            prompt = prompt[0].get(self.content_key)
            if prompt is None:
                return None
        return [{"role": "user", "content": prompt}, {"role": "assistant", "content": resp}]


@dataclass(frozen=True)
class DatasetSpec:
    hf_id: str
    revision: str
    adapter: Adapter
    metadata_columns: tuple[str, ...] = ()
    subset: str | tuple[str, ...] = ""  # one config name, or several read one after another
    splits: tuple[str, ...] = ("train",)


_OPENHERMES = Adapter(conversation_column="conversations", role_key="from", content_key="value",
                      role_values=(("human", "user"), ("gpt", "assistant")))

# The datasets of the reference's chat / tool-use SFT registry: identifiers, pinned revisions, row
# layouts and metadata columns are the datasets' own facts, kept as they are.
DATASETS: dict[str, DatasetSpec] = {
    "allenai/tulu-3-sft-mixture": DatasetSpec("allenai/tulu-3-sft-mixture", "55e9fd6", Adapter(),
                                              ("dataset", "id", "source")),
    "allenai/tulu-v2-sft-mixture": DatasetSpec("allenai/tulu-v2-sft-mixture", "6248b17", Adapter(), ("dataset", "id")),
    "allenai/tulu-v2-sft-mixture-olmo-4096": DatasetSpec("allenai/tulu-v2-sft-mixture-olmo-4096", "7a7c388",
                                                         Adapter(), ("dataset", "id")),
    "sherryy/tulu-3-sft-personas-instruction-following-expanded": DatasetSpec(
        "sherryy/tulu-3-sft-personas-instruction-following-expanded", "79ab2c4", Adapter(), ("dataset", "id")),
    "meta-math/MetaMathQA": DatasetSpec("meta-math/MetaMathQA", "aa4f34d",
                                        Adapter("instruction_response", prompt_column="query",
                                                response_column="response"), ("type",)),
    "openbmb/UltraInteract_sft": DatasetSpec("openbmb/UltraInteract_sft", "2b102e4",
                                             Adapter("instruction_response", prompt_column="instruction",
                                                     response_column="response"), ("task", "dataset")),
    "teknium/OpenHermes-2.5": DatasetSpec("teknium/OpenHermes-2.5", "b820378", _OPENHERMES,
                                          ("id", "category", "source")),
    "HuggingFaceH4/no_robots": DatasetSpec("HuggingFaceH4/no_robots", "e6f9a4a", Adapter(), ("category", "prompt_id")),
    "facebook/natural_reasoning": DatasetSpec("facebook/natural_reasoning", "99eea5d",
                                              Adapter("instruction_list_response", prompt_column="question",
                                                      response_column="responses", content_key="response"),
                                              ("reference_answer",)),
    "smoltalk2-xlam": DatasetSpec("HuggingFaceTB/smoltalk2", "fc6cc21", Adapter(), (), "SFT",
                                  ("xlam_traces_no_think",)),
    "smoltalk2-hermes-fc": DatasetSpec("HuggingFaceTB/smoltalk2", "fc6cc21", Adapter(), (), "SFT",
                                       ("hermes_function_calling_v1_no_think",)),
    "smoltalk2-smolagents": DatasetSpec("HuggingFaceTB/smoltalk2", "fc6cc21", Adapter(), (), "SFT",
                                        ("smolagents_toolcalling_traces_think",)),
}
_OMR_META = ("expected_answer", "problem_source", "problem_type", "generation_model", "inference_mode",
             "pass_rate_72b_tir", "used_in_kaggle")
_GT_META = ("question_id", "question_url", "reference_answer", "model_name", "question_source", "task")
_DOLPHIN_META = ("score", "refusal", "compliance_rating", "overall_quality")
# Further entries of the full chat / reasoning SFT registry (tunix-delphi-rl/sft_data/
# instruction_datasets_marin_original.py).
DATASETS.update({
    "TIGER-Lab/AceCode-89K": DatasetSpec(
        "TIGER-Lab/AceCode-89K", "13216309a9f6cb40b60cb1a9750071efeac414ad",
        Adapter("instruction_response", prompt_column="question", response_column="inferences",
                content_key="completion", best_of="pass_rate"), ("id", "source")),
    "cognitivecomputations/dolphin-r1-nonreasoning": DatasetSpec(
        "cognitivecomputations/dolphin-r1", "f6ac651", Adapter(), _DOLPHIN_META, "nonreasoning"),
    "cognitivecomputations/dolphin-r1-reasoning": DatasetSpec(
        "cognitivecomputations/dolphin-r1", "f6ac651",
        Adapter("message_list_response", prompt_column="messages", response_column="answer"), _DOLPHIN_META,
        ("reasoning-deepseek", "reasoning-flash")),
    "open-r1/OpenThoughts-114k-math": DatasetSpec("open-r1/OpenThoughts-114k-math", "2db609d", Adapter(),
                                                  ("system", "source", "generated_token_count", "correct")),
    "bespokelabs/Bespoke-Stratos-17k": DatasetSpec(
        "bespokelabs/Bespoke-Stratos-17k", "9e9adba",
        Adapter(conversation_column="conversations", role_key="from", content_key="value")),
    "HuggingFaceTB/smoltalk": DatasetSpec("HuggingFaceTB/smoltalk", "2c849df", Adapter(), ("source",), "all"),
    "PrimeIntellect/verifiable-math-problems": DatasetSpec(
        "PrimeIntellect/verifiable-math-problems", "2ad7c92",
        Adapter("instruction_response", prompt_column="prompt", response_column="gold_standard_solution"),
        ("source", "task_type", "problem_id")),
    "GeneralReasoning/GeneralThought-195K-modelanswer": DatasetSpec(
        "GeneralReasoning/GeneralThought-195K", "64f7cb8",
        Adapter("instruction_response", prompt_column="question", response_column="model_answer"), _GT_META),
    "GeneralReasoning/GeneralThought-195K-modelreasoning": DatasetSpec(
        "GeneralReasoning/GeneralThought-195K", "64f7cb8",
        Adapter("instruction_response", prompt_column="question", response_column="model_reasoning"), _GT_META),
    "open-thoughts/OpenThoughts3-1.2M": DatasetSpec("open-thoughts/OpenThoughts3-1.2M", "61bcf9d", _OPENHERMES,
                                                    ("difficulty", "source", "domain")),
    **{f"nvidia/OpenMathReasoning/{sp}": DatasetSpec(
        "nvidia/OpenMathReasoning", "d3d0866",
        Adapter("instruction_response", prompt_column="problem", response_column="generated_solution"), _OMR_META,
        "", (sp,)) for sp in ("cot", "tir", "genselect")},
})
TULU = ("allenai/tulu-3-sft-mixture", "allenai/tulu-v2-sft-mixture", "allenai/tulu-v2-sft-mixture-olmo-4096",
        "sherryy/tulu-3-sft-personas-instruction-following-expanded")
TOOLUSE = ("smoltalk2-xlam", "smoltalk2-hermes-fc", "smoltalk2-smolagents")
DEFAULT_MIX = {"allenai/tulu-3-sft-mixture": 0.85, **{n: 0.05 for n in TOOLUSE}}


def transform_row(row: dict, spec: DatasetSpec) -> dict | None:
    msgs = spec.adapter.to_messages(row)
    if msgs is None:
        return None
    reps = dict(spec.adapter.replacements) if spec.adapter.replacements is not None else THINK_TAGS
    for m in msgs:
        if isinstance(m["content"], str):
            for a, b in reps.items():
                m["content"] = m["content"].replace(a, b)
    meta = {c: row.get(c, "") for c in spec.metadata_columns}
    if spec.adapter.extra_metadata is not None:
        meta.update(spec.adapter.extra_metadata(row) or {})
    return {"messages": msgs, "metadata": meta}


def _read_file(path: str) -> Iterator[dict]:
    if path.endswith(".parquet"):
        import pyarrow.parquet as pq

        pf = pq.ParquetFile(path)
        for batch in pf.iter_batches(batch_size=1024):
            yield from batch.to_pylist()
        return
    opener = gzip.open if path.endswith(".gz") else open
    with opener(path, "rt", encoding="utf-8") as f:
        if path.endswith(".json"):
            data = json.load(f)
            yield from (data if isinstance(data, list) else [data])
            return
        for line in f:
            if line.strip():
                yield json.loads(line)


def snapshot_dir(root: str, spec: DatasetSpec) -> str:
    return os.path.join(root, spec.hf_id)


def iter_rows(root: str, spec: DatasetSpec, split: str | None = None) -> Iterator[dict]:
    """Raw rows of ``spec`` from its local snapshot: files under ``<root>/<hf id>/[<subset>/]`` (each
    subset in turn when there are several) whose path contains the split name (when the snapshot has
    per-split files), in sorted order."""
    root_dir = snapshot_dir(root, spec)
    subsets = (spec.subset,) if isinstance(spec.subset, str) else tuple(spec.subset)
    for sub in subsets:
        base = root_dir
        if sub and os.path.isdir(os.path.join(base, sub)):
            base = os.path.join(base, sub)
        elif sub and len(subsets) > 1:
            raise FileNotFoundError(f"no local snapshot of {spec.hf_id} config {sub!r} under {root_dir}")
        if not os.path.isdir(base):
            raise FileNotFoundError(f"no local snapshot of {spec.hf_id} at {base} (rows are read from local files)")
        files = sorted(p for ext in ("parquet", "jsonl", "jsonl.gz", "json")
                       for p in glob.glob(os.path.join(base, "**", f"*.{ext}"), recursive=True))
        for sp in ([split] if split else spec.splits):
            chosen = [p for p in files if sp in os.path.relpath(p, base)] or (files if len(spec.splits) == 1 else [])
            for p in chosen:
                yield from _read_file(p)


def load_messages(name: str, root: str, limit: int | None = None, split: str | None = None) -> Iterator[dict]:
    spec = DATASETS[name]
    n = 0
    for row in iter_rows(root, spec, split):
        out = transform_row(row, spec)
        if out is None:
            continue
        out["metadata"].setdefault("source_dataset", name)
        yield out
        n += 1
        if limit is not None and n >= limit:
            return


def interleave(streams: dict[str, Iterable[dict]], weights: dict[str, float], seed: int = 0,
               limit: int | None = None) -> Iterator[dict]:
    if not weights or any(w < 0 for w in weights.values()) or not any(weights.values()):
        raise ValueError("interleave needs non-negative weights with a positive sum")
    rng = random.Random(seed)
    live = {k: iter(streams[k]) for k in weights if weights[k] > 0}
    n = 0
    while live:
        names = list(live)
        pick = rng.choices(names, weights=[weights[k] for k in names])[0]
        try:
            row = next(live[pick])
        except StopIteration:
            del live[pick]
            continue
        yield row
        n += 1
        if limit is not None and n >= limit:
            return


def chat_tooluse_mixture(root: str, weights: dict[str, float] | None = None, seed: int = 0,
                         limit: int | None = None) -> Iterator[dict]:
    w = dict(weights or DEFAULT_MIX)
    return interleave({k: load_messages(k, root) for k in w}, w, seed, limit)


def write_messages_jsonl(rows: Iterable[dict], path: str) -> int:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    n = 0
    with open(path, "w") as f:
        for r in rows:
            f.write(json.dumps(r) + "\n")
            n += 1
    return n


def source_counts(rows: Iterable[dict]) -> dict[str, int]:
    counts: dict[str, int] = {}
    for r in rows:
        k = r.get("metadata", {}).get("source_dataset", "?")
        counts[k] = counts.get(k, 0) + 1
    return counts
