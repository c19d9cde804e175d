"""Re-entrant (looped) grug MoE on CPU: R = 1 equals the plain stack, zero-initialised FiLM /
depth bias keep it identical, the extra loss terms are present and differentiable, the learned
router logit bias gets a gradient, and depth sampling stays within the choices."""

import random

import pytest
import torch

from marin_experiments_b200.config import GrugModelConfig
from marin_experiments_b200.models.grug import Transformer
from marin_experiments_b200.models.looped import LoopedConfig, LoopedTransformer

M = GrugModelConfig(vocab_size=256, hidden_dim=64, intermediate_dim=128, shared_expert_intermediate_dim=128,
                    num_experts=4, num_experts_per_token=2, num_layers=4, num_heads=2, num_kv_heads=2, head_dim=32,
                    max_seq_len=32, sliding_window=32)
TOK = torch.randint(0, 256, (2, 32), generator=torch.Generator().manual_seed(0))


def test_r1_matches_plain_stack():
    plain = Transformer(M).init_weights(3)
    lp = LoopedTransformer(LoopedConfig(model=M, num_prelude_layers=1, num_coda_layers=1, iteration_film=True,
                                        depth_conditioned_routing=True)).init_weights(3)
    la, _ = plain.next_token_loss(TOK)
    lb, _ = lp.next_token_loss(TOK)
    assert torch.allclose(la, lb, atol=1e-6)


def test_looped_terms_and_gradients():
    lc = LoopedConfig(model=M, num_prelude_layers=1, num_coda_layers=1, recurrence_steps=3, iteration_film=True,
                      depth_conditioned_routing=True, core_consistency_weight=0.1, anytime_supervision=True,
                      ponder_halting=True)
    m = LoopedTransformer(lc).init_weights(1)
    assert lc.effective_depth() == 1 + 2 * 3 + 1
    loss, met = m.next_token_loss(TOK)
    for k in ("train/core_consistency", "train/anytime_ce", "train/ponder_ce", "train/ponder_kl",
              "train/ponder_expected_steps"):
        assert k in met and torch.isfinite(met[k])
    loss.backward()
    for p in (m.film_scale, m.film_shift, m.depth_bias, m.halt_head):
        assert p.grad is not None and torch.isfinite(p.grad).all()
    assert m.depth_bias.grad.abs().sum() > 0
    # deeper than trained: the last FiLM / bias entry is reused
    l4, _ = m.next_token_loss(TOK, recurrence=5)
    assert torch.isfinite(l4)


def test_randomized_recurrence():
    lc = LoopedConfig(model=M, num_prelude_layers=1, num_coda_layers=1, recurrence_steps=2,
                      randomize_recurrence=True, recurrence_choices=(1, 2, 4))
    m = LoopedTransformer(lc)
    rng = random.Random(0)
    seen = {m.sample_recurrence(rng) for _ in range(50)}
    assert seen == {1, 2, 4} and lc.table_depth == 4
    with pytest.raises(ValueError):
        LoopedConfig(model=M, randomize_recurrence=True)
    with pytest.raises(ValueError):
        LoopedConfig(model=M, num_prelude_layers=3, num_coda_layers=2)


def test_trainer_with_looped_model():
    from marin_experiments_b200.config import GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    lc = LoopedConfig(model=M, num_prelude_layers=1, num_coda_layers=1, recurrence_steps=2, iteration_film=True,
                      depth_conditioned_routing=True, randomize_recurrence=True, recurrence_choices=(1, 2, 3))
    run = GrugRunConfig(model=M, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=5)))
    tr = Trainer(run, device="cpu", model_factory=lambda cfg, local: LoopedTransformer(lc))
    groups = {n: [i.name for i in g["infos"]] for n, g in tr.opt.groups.items()}
    assert "film_scale" in groups["adam"] and "depth_bias" in groups["adam"]
    assert float(tr.store.master_view(tr.store.by_name["film_scale"]).abs().sum()) == 0.0
    losses = [float(tr.train_step({"tokens": TOK})["train/loss"]) for _ in range(4)]
    assert all(l == l for l in losses)
    assert float(tr.store.master_view(tr.store.by_name["film_scale"]).abs().sum()) > 0


def test_depth_sweep_and_tagged_eval():
    from marin_experiments_b200.config import GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.eval import evaluate, evaluate_at_depths, evaluate_tagged
    from marin_experiments_b200.train.trainer import Trainer

    lc = LoopedConfig(model=M, num_prelude_layers=1, num_coda_layers=1, recurrence_steps=2, iteration_film=True,
                      randomize_recurrence=True, recurrence_choices=(1, 2, 3))
    run = GrugRunConfig(model=M, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=5)))
    tr = Trainer(run, device="cpu", model_factory=lambda cfg, local: LoopedTransformer(lc))
    for _ in range(2):
        tr.train_step({"tokens": TOK})
    g = torch.Generator().manual_seed(5)
    web = [{"tokens": torch.randint(0, 256, (2, 32), generator=g)} for _ in range(2)]
    code = [{"tokens": torch.randint(0, 256, (2, 32), generator=g)}]
    res = evaluate_at_depths(tr, web, (1, 2, 3))
    assert set(res) == {1, 2, 3} and "eval/R2/loss" in res[2]
    assert res[1]["eval/R1/loss"] != res[3]["eval/R3/loss"]  # the loop count changes the function
    with torch.no_grad():
        direct = evaluate(tr, web, model_kwargs={"recurrence": 3})["eval/loss"]
    assert abs(direct - res[3]["eval/R3/loss"]) < 1e-6
    tagged = evaluate_at_depths(tr, {"web": web, "code": code}, (2,))[2]
    lw, lc_ = tagged["eval/R2/web/loss"], tagged["eval/R2/code/loss"]
    assert abs(tagged["eval/R2/macro_loss"] - (lw + lc_) / 2) < 1e-9
    assert abs(tagged["eval/R2/micro_loss"] - (2 * lw + lc_) / 3) < 1e-9
    plain = evaluate_tagged(tr, {"web": web}, prefix="x")
    assert set(plain) == {"x/web/loss", "x/macro_loss", "x/micro_loss"}


def test_reentrant_launcher_trains_looped_variant(tmp_path, monkeypatch):
    """The launcher's looped config reaches the trainer (a LoopedTransformer is built and trained)."""
    from marin_experiments_b200.config import DataConfig
    from marin_experiments_b200.experiments import reentrant
    from marin_experiments_b200.experiments.common import GrugLaunchConfig, run_inline
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train import trainer as T

    lc = LoopedConfig(model=M, num_prelude_layers=1, num_coda_layers=1, recurrence_steps=2, iteration_film=True)
    built = []
    orig = T.Trainer._build

    def spy(self):
        orig(self)
        built.append(type(self.model).__name__)

    monkeypatch.setattr(T.Trainer, "_build", spy)
    cfg = GrugLaunchConfig(model=M, looped=lc, data=DataConfig(source="synthetic"), output_path=str(tmp_path),
                           run_id="loop", steps=2, batch_size=2, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                           mp="params=float32,compute=float32,output=float32", save_interval_s=1e9)
    try:
        run_inline(cfg)
    except Exception as e:  # the native data loader is part of the package build
        if "runtime" not in str(e).lower() and "_mxrt" not in str(e):
            raise
        pytest.skip(f"native runtime unavailable: {e}")
    assert built == ["LoopedTransformer"]
    monkeypatch.setenv("GRUG_EXPERIMENT", "e0,e3,e64")
    names = [s.name for s in reentrant.build_steps()]
    assert names == ["grug/reentrant_e0", "grug/reentrant_e3", "grug/reentrant_e64"]
    exps = reentrant.experiments()
    assert exps["e3"][1].recurrence_choices == (2, 4, 8) and exps["e64"][1].anytime_supervision
    assert exps["e0"][1] is None and exps["e1"][1].effective_depth() == exps["e0"][0].num_layers
    with pytest.raises(KeyError, match="unknown experiment"):
        reentrant.build_steps(["e9"])
