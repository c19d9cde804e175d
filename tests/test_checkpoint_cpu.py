"""Checkpoint layout, save/restore round trip, restore search with fallback, temporary/permanent
policy and weights-only initialisation -- on the tiny dense CPU configuration (2 layers, hidden
128, 4 heads of 32, SwiGLU 512, vocab 128256, seq 256, AdamW 3e-4)."""

import json
import os

import pytest
import torch

from marin_experiments_b200.config import CheckpointerConfig, GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
from marin_experiments_b200.optim import AdamConfig
from marin_experiments_b200.train.checkpoint import (Checkpointer, CorruptCheckpointError, checkpoint_candidates,
                                                     initialize_from, load_checkpoint, restore_from_checkpoint,
                                                     save_checkpoint)
from marin_experiments_b200.train.trainer import Trainer

TINY = GrugModelConfig(vocab_size=128256, hidden_dim=128, intermediate_dim=512, num_experts=0, num_layers=2,
                       num_heads=4, num_kv_heads=4, head_dim=32, max_seq_len=256, sliding_window=256,
                       gated_norm=False, qk_norm=False, xsa=False, head_gate=False, shared_expert_intermediate_dim=0)


def _trainer(seed=0, steps=20):
    run = GrugRunConfig(model=TINY, optimizer=AdamConfig(learning_rate=3e-4, warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=steps, seed=seed)))
    return Trainer(run, device="cpu")


def _batch():
    g = torch.Generator().manual_seed(0)
    return {"tokens": torch.randint(0, 128256, (8, 256), generator=g)}


@pytest.fixture(scope="module")
def trained():
    tr = _trainer()
    b = _batch()
    losses = [float(tr.train_step(b)["train/loss"]) for _ in range(20)]
    return tr, losses


def test_tiny_dense_trains(trained):
    _, losses = trained
    assert losses[-1] < losses[0]


def test_save_reload_roundtrip(trained, tmp_path):
    tr, _ = trained
    path = str(tmp_path / "ckpt" / "step-20")
    save_checkpoint(tr, path)
    assert os.path.exists(os.path.join(path, "metadata.json"))
    meta = json.load(open(os.path.join(path, "metadata.json")))
    assert meta["step"] == 20 and meta["is_temporary"] is False
    assert os.path.exists(os.path.join(path, "params", "token_embed.bin")) or any(
        f.startswith("params") for f in os.listdir(path))
    fresh = _trainer(seed=1)
    assert not torch.equal(fresh.store.master, tr.store.master)
    step = load_checkpoint(fresh, path)
    assert step == 20 and fresh.step == 20
    assert torch.equal(fresh.store.master, tr.store.master)
    assert torch.equal(fresh.opt.m, tr.opt.m) and torch.equal(fresh.opt.v, tr.opt.v)
    assert fresh.opt.step_count == tr.opt.step_count
    # both continue identically
    b = _batch()
    la = float(tr.train_step(b)["train/loss"])
    lb = float(fresh.train_step(b)["train/loss"])
    assert la == lb
    assert torch.equal(fresh.store.master, tr.store.master)


def test_restore_search_falls_back(trained, tmp_path):
    tr, _ = trained
    root = str(tmp_path / "ck")
    save_checkpoint(tr, os.path.join(root, "step-5"), step=5)
    save_checkpoint(tr, os.path.join(root, "step-9"), step=9)
    # newest is incomplete (no metadata) -> ignored; next newest is corrupted -> falls back
    os.makedirs(os.path.join(root, "step-12"))
    assert checkpoint_candidates([root])[:2] == [os.path.join(root, "step-9"), os.path.join(root, "step-5")]
    leaf = os.path.join(root, "step-9", "params")
    victim = next(os.path.join(dp, f) for dp, _, fs in os.walk(leaf) for f in fs)
    with open(victim, "r+b") as f:
        f.write(b"\x00\x01\x02\x03")
    fresh = _trainer(seed=2)
    with pytest.raises(CorruptCheckpointError):
        load_checkpoint(fresh, os.path.join(root, "step-9"))
    got = restore_from_checkpoint(fresh, [root])
    assert got == os.path.join(root, "step-5") and fresh.step == 5
    assert restore_from_checkpoint(_trainer(), [str(tmp_path / "none")]) is None
    with pytest.raises(FileNotFoundError):
        restore_from_checkpoint(_trainer(), [str(tmp_path / "none")], load_checkpoint_setting=True)
    assert restore_from_checkpoint(_trainer(), [root], load_checkpoint_setting=False) is None


def test_legacy_train_state_prefix(trained, tmp_path):
    tr, _ = trained
    path = str(tmp_path / "legacy")
    save_checkpoint(tr, path)
    man = json.load(open(os.path.join(path, "manifest.json")))
    man["leaves"] = {"train_state/" + k: v for k, v in man["leaves"].items()}
    json.dump(man, open(os.path.join(path, "manifest.json"), "w"))
    fresh = _trainer(seed=3)
    load_checkpoint(fresh, path)
    assert torch.equal(fresh.store.master, tr.store.master)


def test_initialize_from_weights_only(trained, tmp_path):
    tr, _ = trained
    root = str(tmp_path / "graft")
    save_checkpoint(tr, os.path.join(root, "step-20"))
    fresh = _trainer(seed=4)
    initialize_from(fresh, root)
    assert fresh.step == 0 and fresh.opt.step_count == 0
    assert torch.equal(fresh.store.master, tr.store.master)
    assert float(fresh.opt.m.abs().sum()) == 0.0


def test_checkpointer_policy(trained, tmp_path):
    tr, _ = trained
    now = [0.0]
    cfg = CheckpointerConfig(base_path=str(tmp_path / "perm"), temporary_base_path=str(tmp_path / "tmp"),
                             save_interval_s=10, keep_last_temporary_checkpoints=2, keep=({"every": 4},))
    ck = Checkpointer(cfg, clock=lambda: now[0], background=True)
    for step in range(1, 10):
        now[0] += 6  # a temporary save every other step
        ck.on_step(tr, step)
    ck.on_end(tr)
    perm = sorted(os.listdir(tmp_path / "perm"))
    tmp = sorted(os.listdir(tmp_path / "tmp"))
    assert "step-4" in perm and "step-8" in perm
    assert len(tmp) == 2  # rolling temporaries pruned to the newest two
    assert all(json.load(open(tmp_path / "tmp" / d / "metadata.json"))["is_temporary"] for d in tmp)
    assert restore_from_checkpoint(_trainer(), ck.search_paths()) is not None
