"""Whole-model check: the grug MoE and dense models on the sm_100a path vs the fp32 CPU oracle.

Both start from identical weights (the CPU store's masters loaded into the GPU store); loss and
every parameter's gradient are compared after one forward/backward.
"""

import pytest
import torch

from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
from marin_experiments_b200.optim import GrugMoeAdamHConfig
from marin_experiments_b200.train.trainer import Trainer

pytestmark = pytest.mark.gpu

MOE = GrugModelConfig(vocab_size=2048, hidden_dim=256, intermediate_dim=256, shared_expert_intermediate_dim=512,
                      num_experts=8, num_experts_per_token=2, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                      max_seq_len=256, sliding_window=256, capacity_factor=2.0)
DENSE = GrugModelConfig(vocab_size=2048, hidden_dim=256, intermediate_dim=512, num_experts=0, num_layers=2,
                        num_heads=4, num_kv_heads=4, max_seq_len=256, gated_norm=False, qk_norm=False, xsa=False,
                        head_gate=False, glu=True)


def _pair(cfg):
    run = GrugRunConfig(model=cfg, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10)))
    cpu = Trainer(run, device="cpu")
    gpu = Trainer(run, device="cuda:0")
    gpu.store.load_state_dict(cpu.store.state_dict())
    return cpu, gpu


@pytest.mark.parametrize("cfg", [MOE, DENSE], ids=["moe", "dense"])
def test_model_loss_and_grads(cfg):
    cpu, gpu = _pair(cfg)
    tok = torch.randint(0, cfg.vocab_size, (2, 256), generator=torch.Generator().manual_seed(0))
    lc, _ = cpu.model.next_token_loss(tok, z_loss_weight=1e-4)
    lc.backward()
    lg, _ = gpu.model.next_token_loss(tok.cuda(), z_loss_weight=1e-4)
    lg.backward()
    torch.cuda.synchronize()
    assert abs(lg.item() - lc.item()) < 1e-2 * lc.item()
    bad = []
    for info in cpu.store.infos:
        if not info.trainable:
            continue
        gc = cpu.store.grad_view(info)
        gg = gpu.store.grad_view(info).cpu()
        if gc.norm() < 1e-8:
            continue
        r = ((gg - gc).norm() / gc.norm()).item()
        # routed expert weights see the discrete top-k decisions: a few near-tied tokens route
        # differently under bf16 activations than under the fp32 oracle
        tol = 0.15 if (".mlp.w_" in info.name and info.ndim == 3) else 6e-2
        if r > tol:
            bad.append((info.name, r))
    assert not bad, bad


def test_train_steps_decrease_loss():
    _, gpu = _pair(MOE)
    tok = torch.randint(0, MOE.vocab_size, (4, 256), generator=torch.Generator().manual_seed(1)).pin_memory()
    losses = [float(gpu.train_step({"tokens": tok})["train/loss"].item()) for _ in range(6)]
    assert losses[-1] < losses[0], losses


def test_optimizer_step_matches_cpu():
    """One AdamH/Adam step on identical gradients: GPU kernels vs the CPU implementation."""
    cpu, gpu = _pair(MOE)
    g = torch.randn(cpu.store.numel, generator=torch.Generator().manual_seed(3)) * 1e-2
    cpu.store.grad.copy_(g)
    gpu.store.grad.copy_(g.cuda())
    cpu.opt.step()
    gpu.opt.step()
    torch.cuda.synchronize()
    d = (gpu.store.master.cpu() - cpu.store.master)
    assert d.abs().max().item() < 1e-5, d.abs().max().item()


@pytest.mark.parametrize("mode", ["recompute_all", "save_moe"])
def test_remat_matches_no_remat_gpu(mode):
    """Activation recompute on the sm_100a path: same loss and gradients as keeping every
    activation, and a lower allocator high-water mark for the same microbatch."""
    import dataclasses

    tok = torch.randint(0, MOE.vocab_size, (4, 256), generator=torch.Generator().manual_seed(2))
    out = {}
    for m in ("none", mode):
        cfg = dataclasses.replace(MOE, remat_mode=m, num_layers=4)
        run = GrugRunConfig(model=cfg, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                            trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10)))
        tr = Trainer(run, device="cuda:0", micro_batch=4)
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        lg, _ = tr.model.next_token_loss(tok.cuda(), z_loss_weight=1e-4)
        lg.backward()
        torch.cuda.synchronize()
        out[m] = (lg.item(), tr.store.grad.clone(), torch.cuda.max_memory_allocated() - base)
        del tr, lg
    (l0, g0, m0), (l1, g1, m1) = out["none"], out[mode]
    assert abs(l1 - l0) < 1e-4 * abs(l0)
    assert ((g1 - g0).norm() / g0.norm()).item() < 1e-3
    assert m1 < m0, (m0, m1)


@pytest.mark.parametrize("corrector,tau,damp", [("none", 2, 1.0), ("dc_asgd", 2, 1.0), ("dc_asgd_ema", 1, 1.0),
                                                ("wp_preorth", 2, 1.0), ("lr_damp", 1, 0.5)])
def test_delayed_step_fused_matches_cpu(corrector, tau, damp):
    """The delayed-gradient step as two sm_100a passes around the fused AdamH vs the torch
    implementation on CPU: same weights, last update and raw momentum after 4 steps of identical
    gradients (per-stage delays: the embedding stalest, the head fresh)."""
    from marin_experiments_b200.optim.delayed import DelayedGrugMoeAdamHConfig

    opt = DelayedGrugMoeAdamHConfig(warmup=0.0, tau=tau, corrector=corrector, lr_damp=damp, num_stages=1 + tau,
                                    num_layers=MOE.num_layers)
    run = GrugRunConfig(model=MOE, optimizer=opt, trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10)))
    cpu = Trainer(run, device="cpu")
    gpu = Trainer(run, device="cuda:0")
    gpu.store.load_state_dict(cpu.store.state_dict())
    gen = torch.Generator().manual_seed(4)
    for _ in range(4):
        g = torch.randn(cpu.store.numel, generator=gen) * 1e-2
        cpu.store.grad.copy_(g)
        gpu.store.grad.copy_(g.cuda())
        cpu.opt.step()
        gpu.opt.step()
    torch.cuda.synchronize()
    assert (gpu.store.master.cpu() - cpu.store.master).abs().max().item() < 1e-5
    assert (gpu.opt.last_update.cpu() - cpu.opt.last_update).abs().max().item() < 1e-5
    if cpu.opt.m_raw is not None:
        assert (gpu.opt.m_raw.cpu() - cpu.opt.m_raw).abs().max().item() < 1e-6
    # the bf16 compute copy follows the (damped) masters
    assert (gpu.store.compute.float() - gpu.store.master.to(torch.bfloat16).float()).abs().max().item() == 0
