"""MoE calculator: its formulas (shared by the HTML page) equal the framework's FLOP and parameter
accounting, and the committed page is the current rendering."""

import dataclasses
import os

from marin_experiments_b200.parallel.pipeline_entry import megagpt_model
from marin_experiments_b200.utils import flops, moe_calculator as mc
from marin_experiments_b200.utils.perf_model import param_split


def _check(cfg):
    v = mc.evaluate(mc.inputs_from_config(cfg, TPS=1.0e5, GPUS=2, PEAK=2.25e15, HOURS=1))
    c = flops.fwd_components(cfg)
    close = lambda a, b: abs(a - b) <= 1e-9 * max(abs(b), 1.0)  # noqa: E731
    assert close(v["f_attn_proj"], c["attn_proj_QKVO"]) and close(v["f_attn_scores"], c["attn_scores_AV"])
    assert close(v["f_routed"], c["routed_experts"]) and close(v["f_shared"], c["shared_expert"])
    assert close(v["f_dense"], c["dense_mlp"]) and close(v["f_gated"], c["gated_norms"])
    assert close(v["f_head"], c["lm_head"]) and close(v["fwd"], c["_total"])
    assert close(v["train"], flops.training_flops_per_token(cfg))
    assert close(v["mfu"], flops.mfu(1.0e5, cfg, 2))
    experts, other = param_split(cfg)
    assert close(v["p_experts"], experts) and close(v["p_total"], experts + other)
    if cfg.num_experts:
        assert close(v["p_active"], experts * cfg.num_experts_per_token / cfg.num_experts + other)
    return v


def test_formulas_match_accounting():
    cfg = megagpt_model()
    v = _check(cfg)
    assert 5.5e9 < v["p_total"] < 6.5e9 and v["tokens"] == 1.0e5 * 3600
    _check(dataclasses.replace(cfg, embed_dim=512))  # factorized embedding
    _check(dataclasses.replace(cfg, num_experts=0, num_experts_per_token=0, intermediate_dim=4096,
                               shared_expert_intermediate_dim=0))  # dense


def test_expressions_are_python_and_javascript():
    # only the shared subset: names, numbers, + - * / ( ) and comparisons as 0/1 factors
    allowed = set("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ_0123456789.+-*/()<>=! ")
    for _, _, expr in mc.FORMULAS:
        assert set(expr) <= allowed, expr
        assert "**" not in expr and "//" not in expr and " and " not in expr and " or " not in expr


def test_committed_page_is_current():
    path = os.path.join(os.path.dirname(mc.__file__), "moe_calculator.html")
    cfg = megagpt_model()
    page = mc.render(mc.inputs_from_config(cfg, TPS=662754, GPUS=8, PEAK=2.25e15, HOURS=24))
    assert open(path).read() == page
    assert "<script src" not in page and "http" not in page.split("<script>")[1]
    for _, _, expr in mc.FORMULAS:
        assert expr in page
