"""Tiny template pipeline: corpus -> tokenize -> train -> checkpoint (tiny-stories/launch.py:116-260).

The corpus step stands in for the Hugging Face download (there is no network): it copies the text
files named by ``TINY_STORIES_PATH`` or, without one, writes a small deterministic synthetic story
corpus. The tokenizer is the built-in byte tokenizer (ids < 257 inside the 128,256-entry vocab of
``TINY_MODEL``). CPU runs use fp32 and 1,000 documents, like the reference's CPU smoke settings.

Run: ``python -m marin_experiments_b200.experiments.tiny_stories --prefix /tmp/out [--dry_run]``.
"""

from __future__ import annotations

import glob
import os
import random
import shutil
from dataclasses import dataclass

import torch

from ..config import DataConfig, GrugModelConfig, GrugTrainerConfig
from ..data.tokenize import TokenizeConfig, tokenize
from ..executor import ExecutorStep, executor_main, output_path_of, this_output_path, versioned
from ..optim import AdamConfig
from .common import GrugLaunchConfig, run_inline

# ~30M-parameter template model (ReLU MLP, no GatedNorm / QK-norm / XSA / head gate).
TINY_MODEL = GrugModelConfig(vocab_size=128_256, hidden_dim=128, intermediate_dim=448, num_layers=4, num_heads=2,
                             num_kv_heads=2, max_seq_len=1024, sliding_window=1024, num_experts=0,
                             shared_expert_intermediate_dim=0, gated_norm=False, qk_norm=False, xsa=False,
                             head_gate=False, mlp_activation="relu", glu=False)


def _accelerator() -> str:
    acc = os.environ.get("ACCELERATOR", "").lower()
    return acc if acc in ("cpu", "gpu") else ("gpu" if torch.cuda.is_available() else "cpu")


@dataclass(frozen=True)
class CorpusConfig:
    output_path: str
    source: str | None = None
    num_docs: int = 2000
    seed: int = 0


_WORDS = ("the little dog cat girl boy sun tree happy sad ran jumped played found a big red ball in park "
          "and then they went home because it was late mom said good night friend smiled").split()


def write_corpus(cfg: CorpusConfig) -> None:
    os.makedirs(cfg.output_path, exist_ok=True)
    if cfg.source:
        for f in sorted(glob.glob(os.path.join(cfg.source, "*"))):
            if os.path.isfile(f):
                shutil.copy(f, cfg.output_path)
        return
    rng = random.Random(cfg.seed)
    with open(os.path.join(cfg.output_path, "train.txt"), "w") as f:
        for _ in range(cfg.num_docs):
            n = rng.randint(20, 80)
            f.write("Once upon a time " + " ".join(rng.choice(_WORDS) for _ in range(n)) + ".\n")


def build_steps(steps: int | None = None, batch_size: int | None = None) -> list[ExecutorStep]:
    cpu = _accelerator() == "cpu"
    corpus = ExecutorStep(name="raw/tinystories", fn=write_corpus,
                          config=CorpusConfig(output_path=this_output_path(),
                                              source=os.environ.get("TINY_STORIES_PATH") or None))
    tokenized = ExecutorStep(name="tokenized/tinystories", fn=tokenize,
                             config=TokenizeConfig(train_paths=(output_path_of(corpus),), cache_path=this_output_path(),
                                                   tokenizer=versioned("bytes"), line_docs=True,
                                                   sample_count=versioned(1_000 if cpu else None)))
    model = TINY_MODEL if not cpu else TINY_MODEL.__class__(**{**TINY_MODEL.__dict__, "max_seq_len": 256,
                                                              "sliding_window": 256})
    launch = GrugLaunchConfig(
        model=versioned(model),
        data=DataConfig(source="cache", cache_dir=output_path_of(tokenized), seed=0),
        output_path=this_output_path(), run_id=os.environ.get("GRUG_RUN_ID", f"tiny-stories-30m-{_accelerator()}"),
        steps=versioned(steps or (20 if cpu else 2000)), batch_size=versioned(batch_size or (8 if cpu else 64)),
        seed=versioned(0),
        mp=versioned("params=float32,compute=float32,output=float32" if cpu
                     else "params=float32,compute=bfloat16,output=bfloat16"),
        optimizer=versioned(AdamConfig(learning_rate=6e-4, weight_decay=0.1, lr_schedule="cosine", decay=0.2,
                                       min_lr_ratio=0.1, warmup=0.1 if cpu else 200)),
        grug_trainer=versioned(GrugTrainerConfig(z_loss_weight=1e-4, ema_beta=None, log_every=1)),
        save_interval_s=600, keep=({"every": 1000},), eval=None,
    )
    train = ExecutorStep(name="tiny-stories/tinystories-30m", fn=run_inline, config=launch)
    return [corpus, tokenized, train]


def main(argv=None):
    return executor_main(build_steps(), description=f"tiny-stories: ~30M grug on a local corpus ({_accelerator()})",
                         argv=argv)


if __name__ == "__main__":
    main()
