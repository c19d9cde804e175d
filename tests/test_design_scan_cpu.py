"""Design-space scan / decision table (the analytical next-run sizing tools)."""

from marin_experiments_b200.parallel.pipeline_entry import megagpt_model
from marin_experiments_b200.utils import design_scan as ds
from marin_experiments_b200.utils.perf_model import Layout, estimate


def test_params_and_memory():
    cfg = megagpt_model()
    total, active = ds.params(cfg)
    assert 5.5e9 < total < 6.5e9  # 24 x 64 experts x 3 x 1536 x 768 routed + the dense rest
    assert 0.15 * total < active < 0.25 * total  # K=4 of 64 routed experts + attention, shared expert, embeddings
    # experts shard over the EP group: more GPUs, less memory per GPU
    assert ds.memory_per_gpu(cfg, 8, 32768) < ds.memory_per_gpu(cfg, 2, 32768) < ds.memory_per_gpu(cfg, 1, 32768)
    # one GPU with 16-sequence microbatches does not fit (observed out of memory), 8 sequences do
    assert ds.memory_per_gpu(cfg, 1, 16 * 2048) > ds.HBM_BYTES > ds.memory_per_gpu(cfg, 1, 8 * 2048)


def test_scan_anchor_and_ordering():
    cfg = megagpt_model()
    measured = 662_754.0
    modelled = estimate(cfg, Layout(gpus=8, ep=8, tokens_per_gpu=65536)).tokens_per_s
    rows = ds.scan(ds.DEFAULT_CANDIDATES, anchor=(cfg, measured))
    assert len(rows) == len(ds.DEFAULT_CANDIDATES)
    for r in rows:
        unscaled = estimate(r.cfg, Layout(gpus=8, ep=8, tokens_per_gpu=65536)).tokens_per_s
        assert abs(r.tokens_per_s - unscaled * measured / modelled) < 1e-6 * r.tokens_per_s
        assert r.tokens_per_expert == r.tokens * r.cand.k / r.cand.experts
    by = {r.cand.name: r for r in rows}
    # more experts at the same K: more total parameters and memory, fewer tokens per expert
    assert by["E128/K8"].total > by["E64/K8"].total
    assert by["E128/K8"].tokens_per_expert < by["E64/K8"].tokens_per_expert
    text = ds.table(rows, baseline="E64/K4", min_tokens_per_expert=5e9)
    assert "experts starved" in text and text.count("\n") == len(rows) + 1


def test_decision_table():
    c = ds.DEFAULT_CANDIDATES
    ranked = ds.decision_table([ds.Measured(c[0], 600_000.0, True), ds.Measured(c[2], 500_000.0, True),
                                ds.Measured(c[3], None, False)], hours=24, cooldown_hours=4,
                               min_tokens_per_expert=1e9)
    assert ranked[-1][0] == c[3].name and ranked[-1][3] == "does not fit"
    assert ranked[0][3] == "ok" and ranked[0][1] >= ranked[1][1]
