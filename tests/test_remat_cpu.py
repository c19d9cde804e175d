"""Activation recompute (``remat_mode``): the same loss and gradients as keeping every activation,
for the dense and MoE models on CPU; unknown modes are rejected."""

import dataclasses

import pytest
import torch

MOE = dict(vocab_size=512, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128, num_experts=4,
           num_experts_per_token=2, num_layers=2, num_heads=2, num_kv_heads=2, head_dim=32, max_seq_len=64,
           sliding_window=64, capacity_factor=2.0)
DENSE = dict(vocab_size=512, hidden_dim=64, intermediate_dim=128, num_experts=0, num_layers=2, num_heads=2,
             num_kv_heads=2, head_dim=32, max_seq_len=64, sliding_window=64, shared_expert_intermediate_dim=0)


def _step(cfg_kw, mode, calls=None):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    cfg = GrugModelConfig(**cfg_kw, remat_mode=mode)
    run = GrugRunConfig(model=cfg, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=4, seed=0)))
    tr = Trainer(run, device="cpu", micro_batch=2)
    g = torch.Generator().manual_seed(0)
    tokens = torch.randint(0, 512, (4, 64), generator=g)
    snap = []
    opt_step = tr.opt.step

    def step_with_snapshot():  # the optimizer clears the gradients: keep them first
        snap.append(tr.store.grad.clone())
        opt_step()

    tr.opt.step = step_with_snapshot
    met = tr.train_step({"tokens": tokens})
    grad = snap[0]
    assert grad.abs().sum() > 0
    return float(met["train/loss"]), grad, tr.store.master.clone()


@pytest.mark.parametrize("kw", [MOE, DENSE], ids=["moe", "dense"])
@pytest.mark.parametrize("mode", ["recompute_all", "save_moe"])
def test_remat_matches_no_remat(kw, mode, monkeypatch):
    from marin_experiments_b200.ops import api

    calls = {"attn": 0, "moe": 0}
    attn, moe = api.attention_block, api.moe_experts

    def count_attn(*a, **k):
        calls["attn"] += 1
        return attn(*a, **k)

    def count_moe(*a, **k):
        calls["moe"] += 1
        return moe(*a, **k)

    monkeypatch.setattr(api, "attention_block", count_attn)
    monkeypatch.setattr(api, "moe_experts", count_moe)
    loss0, grad0, p0 = _step(kw, "none")
    base = dict(calls)
    loss1, grad1, p1 = _step(kw, mode)
    # 2 layers x 2 microbatches: every attention runs once more in backward; the routed experts
    # run again only under recompute_all
    assert calls["attn"] - base["attn"] == 2 * base["attn"]
    if kw is MOE:
        assert calls["moe"] - base["moe"] == (2 if mode == "recompute_all" else 1) * base["moe"]
    assert loss1 == pytest.approx(loss0, rel=1e-6)
    assert torch.allclose(grad1, grad0, rtol=1e-5, atol=1e-7)
    assert torch.allclose(p1, p0, rtol=1e-5, atol=1e-7)


def test_unknown_remat_mode_is_rejected():
    from marin_experiments_b200.config import GrugModelConfig

    with pytest.raises(ValueError, match="remat_mode"):
        GrugModelConfig(**MOE, remat_mode="save_everything")
    cfg = GrugModelConfig(**MOE)
    with pytest.raises(ValueError, match="remat_mode"):
        dataclasses.replace(cfg, remat_mode="bogus")
