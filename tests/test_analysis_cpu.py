"""Run analysis: sweep logs, tracker histories, profiler breakdowns."""

import json
import os

from marin_experiments_b200.utils import analysis as an
from marin_experiments_b200.utils.tracker import JsonlTracker

ARM = ("[arm] sw-d1536-e64-k4  mode=fixed D=1536 d_e=1536(factorized=False) seq=2048 E=64 k=4 min_k=0 coef=0.0 "
       "nominal_active_frac=6.2500% batch=256 steps=100 tokens=0.1B layers=24 I_expert=768 "
       "mesh(EP=8,TP=1,replica=None) data=synth budget=1e+19 remat=none moe_impl=ep attn=sm100 curriculum=None\n")


def _thru(steps, tok):
    return "".join(f"[THRUPUT] step={s} dt=0.800s tok_s={tok + s} mfu=0.2100 bs=256\n" for s in steps)


def test_sweep_logs(tmp_path):
    ok = tmp_path / "a.log"
    ok.write_text(ARM + _thru(range(12), 600000))
    oom = tmp_path / "b.log"
    oom.write_text(ARM.replace("sw-d1536-e64-k4", "sw-big") + _thru(range(3), 1)
                   + "torch.OutOfMemoryError: CUDA out of memory. Tried to allocate 2.00 GiB\n")
    nan = tmp_path / "c.log"
    nan.write_text(_thru(range(10), 500000) + "FloatingPointError: loss is nan at step 10\n")
    runs = an.analyze_logs([str(ok), str(oom), str(nan)], warmup=8)
    assert runs[0].arm == {"run": "sw-d1536-e64-k4", "D": 1536, "seq": 2048, "E": 64, "k": 4, "batch": 256,
                           "budget": 1e19}
    assert runs[0].tok_s == 600009.5 and runs[0].n_steps == 4 and runs[0].last_step == 11
    assert runs[0].failure == "" and runs[1].failure == "oom" and runs[2].failure == "nan"
    assert runs[1].tok_s is None and runs[1].last_step == 2
    table = an.sweep_table(runs).splitlines()
    assert "sw-d1536-e64-k4" in table[2] and "600,010" in table[2]
    assert table[-1].rstrip(" |").endswith("oom") or table[-1].rstrip(" |").endswith("nan")
    assert an.classify_failure("x\nNCCL error: unhandled system error\nillegal memory access") == "nccl"


def test_tracker_iso_step(tmp_path):
    for rid, last, loss0 in (("run-a", 50, 5.0), ("run-b", 30, 4.0), ("other", 10, 1.0)):
        t = JsonlTracker(str(tmp_path), rid)
        for s in range(0, last + 1, 10):
            t.log({"train/loss": loss0 - 0.01 * s, "lr": 1e-3}, step=s)
        if rid == "run-a":
            t.log_summary({"train/loss": 4.2})
        t.finish()
    with open(tmp_path / "run-b" / "metrics.jsonl", "a") as f:
        f.write('{"step": 40, "train/lo')  # torn last line from a killed run
    dirs = an.run_dirs(str(tmp_path), "^run-")
    assert [os.path.basename(d) for d in dirs] == ["run-a", "run-b"]
    res = {r["run"]: r for r in an.collect_results(dirs, ["train/loss"])}
    assert res["run-a"]["train/loss"] == 4.2 and res["run-b"]["train/loss"] == 3.7
    assert res["run-b"]["max_step"] == 30
    iso = {r["run"]: r for r in an.iso_step(dirs, 25, ["train/loss"])}
    assert iso["run-a"]["train/loss"] == 4.8 and iso["run-a"]["train/loss@step"] == 20
    assert iso["run-b"]["train/loss@step"] == 20
    assert "run-a" in an.rows_table(list(iso.values()), ["train/loss", "train/loss@step"])
    assert an.main(["iso-step", str(tmp_path), "--step", "25", "--match", "run-"]) is None


def test_profile_breakdown(tmp_path):
    ev = [
        {"ph": "X", "cat": "kernel", "name": "void gemm_sm100_kernel<256, 6, 0, 0, 0, 1>(GemmParams)", "dur": 600.0},
        {"ph": "X", "cat": "kernel", "name": "void gemm_sm100_kernel<128, 4, 0, 1, 3, 0>(GemmParams)", "dur": 200.0},
        {"ph": "X", "cat": "kernel", "name": "void fa_fwd_sm100_kernel<true>(FwdArgs)", "dur": 100.0},
        {"ph": "X", "cat": "kernel", "name": "flash_bwd_prep_kernel", "dur": 20.0},
        {"ph": "X", "cat": "kernel", "name": "ncclDevKernel_AllReduce_Sum_f32_RING_LL", "dur": 50.0},
        {"ph": "X", "cat": "kernel", "name": "ep_dispatch_push_kernel", "dur": 30.0},
        {"ph": "X", "cat": "gpu_memcpy", "name": "Memcpy HtoD (Pinned -> Device)", "dur": 0.0},
        {"ph": "X", "cat": "cpu_op", "name": "aten::mm", "dur": 999.0},
    ]
    path = tmp_path / "t.json"
    path.write_text(json.dumps({"traceEvents": ev}))
    b = an.profile_breakdown(an.load_trace(str(path)), steps=2)
    cats = {c: ms for c, ms, _ in b["categories"]}
    assert abs(b["total_ms_per_step"] - 0.5) < 1e-9
    assert abs(cats["GEMM (tcgen05)"] - 0.4) < 1e-9 and abs(cats["attention backward"] - 0.01) < 1e-9
    assert "collective (NCCL)" in cats and "EP exchange (NVLink peer kernels)" in cats
    assert b["categories"][0][0] == "GEMM (tcgen05)" and b["launches_per_step"] == 3.5
    assert "GEMM (tcgen05)" in an.breakdown_table(b)


def test_profile_call_cpu(tmp_path):
    import torch

    x = torch.randn(64, 64)
    b = an.profile_call(lambda: x @ x, steps=2, trace_path=str(tmp_path / "p.json"))
    assert os.path.exists(tmp_path / "p.json") and b["total_ms_per_step"] >= 0.0


def test_sweep_cli_watch_and_glob(tmp_path, capsys):
    (tmp_path / "r1.log").write_text(ARM + _thru(range(10), 1000))
    an.main(["sweep", str(tmp_path / "*.log"), "--warmup", "8", "--watch", "0.01", "--rounds", "2"])
    out = capsys.readouterr().out
    assert out.count("| run |") == 2 and "sw-d1536-e64-k4" in out


def test_isoloss_token_overhead(tmp_path):
    import pytest

    import json
    import os

    import numpy as np

    from marin_experiments_b200.utils import analysis as A

    steps = np.arange(0, 6001, 20)
    sync = 2.0 + 3.0 * np.exp(-steps / 1000.0)
    slow = 2.0 + 3.0 * np.exp(-steps / 1500.0)  # the same curve, 1.5x more steps to each loss
    floor = 2.3 + 3.0 * np.exp(-steps / 1000.0)  # converged above the reference
    hist = {"sync": list(zip(steps, sync)), "delayed": list(zip(steps, slow)), "floor": list(zip(steps, floor))}
    rows = {r["run"]: r for r in A.isoloss(hist, "sync", tail_frac=0.05, window=5)}
    assert abs(rows["sync"]["gap"]) < 1e-12 and rows["sync"]["overhead"] == pytest.approx(1.0, abs=0.02)
    assert rows["delayed"]["overhead"] == pytest.approx(1.5, rel=0.05) and rows["delayed"]["slope_per_1k"] < 0
    assert rows["floor"]["gap"] == pytest.approx(0.3, abs=0.01)
    sm = A.smooth([1.0, 1.0, 1.0, 1.0], 3)
    assert np.allclose(sm, 1.0)  # ends are not pulled toward zero
    for name, h in hist.items():
        d = tmp_path / name
        os.makedirs(d)
        with open(d / "metrics.jsonl", "w") as f:
            for s, v in h:
                f.write(json.dumps({"step": int(s), "train/loss": float(v)}) + "\n")
    A.main(["isoloss", str(tmp_path), "--sync", "sync", "--tail", "0.05", "--window", "5"])
