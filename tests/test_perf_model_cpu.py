"""The analytical B200 throughput model: scaling trends, pipeline bubbles and exposed comm."""

from marin_experiments_b200.parallel.pipeline_entry import megagpt_model
from marin_experiments_b200.utils.perf_model import Hardware, Layout, estimate, table


def test_trends():
    cfg = megagpt_model()
    hw = Hardware()
    e1 = estimate(cfg, Layout(gpus=1, ep=1), hw)
    e8 = estimate(cfg, Layout(gpus=8, ep=8), hw)
    assert e8.tokens_per_s > 6 * e1.tokens_per_s and e8.tokens_per_s < 8 * e1.tokens_per_s
    assert e1.parts["ep_exchange_s"] == 0 and e8.parts["ep_exchange_s"] > 0
    hidden = estimate(cfg, Layout(gpus=8, ep=8, ep_overlap=1.0), hw)
    assert hidden.exposed_comm_fraction < e8.exposed_comm_fraction
    z = estimate(cfg, Layout(gpus=8, ep=2, pp=4, microbatches=16, schedule="zb"), hw)
    g = estimate(cfg, Layout(gpus=8, ep=2, pp=4, microbatches=16, schedule="gpipe"), hw)
    assert z.parts["pp_bubble_fraction"] < g.parts["pp_bubble_fraction"] and z.step_s < g.step_s
    assert "| 8 |" in table(cfg, [Layout()], hw)
