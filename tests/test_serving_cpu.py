"""Qwen3 serving on CPU: HF export/import round trip with coverage, deterministic greedy generation,
sampling controls, stop strings, and the HTTP API."""

import torch

from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model, load_hf
from marin_experiments_b200.models.qwen3_export import export_hf
from marin_experiments_b200.serving.server import build_app, tiny_engine


def test_hf_roundtrip(tmp_path):
    cfg = Qwen3Config(vocab_size=300, hidden_dim=64, intermediate_dim=128, num_layers=2, num_heads=2, num_kv_heads=1,
                      head_dim=32, rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                 "high_freq_factor": 4.0, "original_max_position_embeddings": 64},
                      max_seq_len=128)
    m = Qwen3Model(cfg).init_weights(1)
    export_hf(m, str(tmp_path / "hf"))
    m2 = load_hf(str(tmp_path / "hf"), dtype=torch.float32)
    tok = torch.randint(0, 300, (2, 20), generator=torch.Generator().manual_seed(0))
    a, b = m.forward_reference(tok), m2.forward_reference(tok)
    assert torch.allclose(a, b, atol=2e-2, rtol=2e-2)  # bf16 storage in the snapshot
    assert (a.argmax(-1) == b.argmax(-1)).float().mean() > 0.95


def test_generate_and_stop():
    eng = tiny_engine("cpu")
    a = eng.generate(["hello", "abc"], max_tokens=8, temperature=0.0)
    b = eng.generate(["hello", "abc"], max_tokens=8, temperature=0.0)
    assert a == b and len(a) == 2
    s1 = eng.generate(["x"], max_tokens=6, temperature=1.0, seed=1)
    s2 = eng.generate(["x"], max_tokens=6, temperature=1.0, seed=1)
    assert s1 == s2
    full = eng.generate(["q"], max_tokens=10, temperature=0.0)[0]
    if len(full) > 2:
        cut = eng.generate(["q"], max_tokens=10, temperature=0.0, stop=[full[1]])[0]
        assert full[1] not in cut and full.startswith(cut)


def test_http_api():
    from fastapi.testclient import TestClient

    client = TestClient(build_app(tiny_engine("cpu"), "tiny"))
    assert client.get("/health").json()["ok"] is True
    r = client.post("/generate", json={"prompt": "hi", "max_tokens": 4, "temperature": 0.0})
    assert r.status_code == 200 and isinstance(r.json()["text"], str)
    r = client.post("/generate", json={"prompts": ["a", "b"], "max_tokens": 3, "temperature": 0.0})
    assert len(r.json()["texts"]) == 2
    assert client.post("/generate", json={"prompt": "a", "prompts": ["b"]}).status_code == 400
    r = client.post("/v1/completions", json={"prompt": "hey", "max_tokens": 3, "temperature": 0.0})
    assert r.json()["object"] == "text_completion" and len(r.json()["choices"]) == 1
    too_long = client.post("/generate", json={"prompt": "hi", "max_tokens": 100000})
    assert too_long.status_code == 400 and "max_len" in too_long.json()["detail"]


def test_http_client_against_live_server():
    import socket
    import threading
    import time

    import uvicorn

    from marin_experiments_b200.serving import client

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    server = uvicorn.Server(uvicorn.Config(build_app(tiny_engine("cpu"), "tiny"), host="127.0.0.1", port=port,
                                           log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{port}"
    try:
        t0 = time.time()
        while not server.started:
            assert time.time() - t0 < 30
            time.sleep(0.05)
        assert client.health(url) == {"ok": True, "model": "tiny"}
        one = client.generate(url, "hi", max_tokens=4, temperature=0.0)
        assert isinstance(one, str) and one == client.generate(url, "hi", max_tokens=4, temperature=0.0)
        assert len(client.generate(url, ["a", "b"], max_tokens=3, temperature=0.0)) == 2
        assert isinstance(client.complete(url, "hey", max_tokens=3, temperature=0.0), str)
        import pytest

        with pytest.raises(client.ServingError, match="HTTP 4"):
            client.generate(url, [], max_tokens=3)
    finally:
        server.should_exit = True
        th.join(timeout=10)


class _ScriptedCalcEngine:
    """Answers the calculator prompt like a perfect policy; records overlapping generate calls."""

    ready = True

    def __init__(self):
        import threading

        self.active = self.peak = 0
        self.mu = threading.Lock()

    def generate(self, prompts, **kw):
        import time

        with self.mu:
            self.active += 1
            self.peak = max(self.peak, self.active)
        time.sleep(0.02)
        outs = []
        for text in prompts:
            q = [ln for ln in text.split("\n") if ln.startswith("Q: ")][-1]
            ops = [int(v) for v in q[3:].split(" * ")]
            res = [int(ln.split(": ")[1]) for ln in text.split(q, 1)[1].split("\n") if ln.startswith("Tool result: ")]
            if not res:
                outs.append(f"CALC({ops[0]} * {ops[1]})")
            elif len(res) < len(ops) - 1:
                outs.append(f"CALC({res[-1]} * {ops[len(res) + 1]})")
            else:
                outs.append(str(res[-1]))
        with self.mu:
            self.active -= 1
        return outs


def test_calc_endpoint_dashboard_and_serialised_engine():
    import threading

    from fastapi.testclient import TestClient

    eng = _ScriptedCalcEngine()
    client = TestClient(build_app(eng, "calc-demo"))
    page = client.get("/")
    assert page.status_code == 200 and "calc-demo" in page.text and 'fetch(url' in page.text
    assert "<script src" not in page.text  # self-contained
    r = client.post("/calc", json={"question": "12 * 34 * 56"}).json()
    assert r["answer"] == str(12 * 34 * 56) and r["calls"] == 2 and r["correct"] is True
    assert r["transcript"].startswith("Q: 12 * 34 * 56\nCALC(12 * 34)\nTool result: 408")
    assert client.post("/calc", json={"question": "Q: 7 * 6"}).json()["answer"] == "42"
    assert client.post("/calc", json={"question": "7 + 6"}).status_code == 400
    assert client.post("/calc", json={"question": "7"}).status_code == 400
    assert client.post("/calc", json={"question": "2 * 3", "max_turns": 10**6}).status_code == 400
    assert client.post("/calc", json={"question": " * ".join(["2"] * 40)}).status_code == 400

    def hit():
        client.post("/calc", json={"question": "3 * 4 * 5"})

    th = [threading.Thread(target=hit) for _ in range(6)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert eng.peak == 1  # generations never overlap on the shared engine


def test_served_model_as_agent_policy(tmp_path):
    """A terminal task solved by a served model: the chat policy renders the conversation, stops at the
    end marker and returns the reply."""
    import json
    import socket
    import threading
    import time

    import uvicorn

    from marin_experiments_b200.data.chat import IM_END
    from marin_experiments_b200.rl import terminal, terminal_tasks
    from marin_experiments_b200.serving import client

    terminal_tasks.write_tasks(str(tmp_path / "tasks"), 2, seed=3)
    tasks = terminal.load_tasks(str(tmp_path / "tasks"))
    acts = {t.instruction: terminal_tasks.oracle_actions(t) for t in tasks}

    class OracleEngine:
        ready = True

        def generate(self, prompts, stop=None, **kw):
            out = []
            for p in prompts:
                inst = next(k for k in acts if k in p)
                n = p.count("<|im_start|>assistant") - 1  # assistant turns already taken
                out.append(acts[inst][n] + IM_END + "trailing text")
                assert stop == [IM_END]
            return out

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    srv = uvicorn.Server(uvicorn.Config(build_app(OracleEngine(), "oracle"), host="127.0.0.1", port=port,
                                       log_level="warning"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    try:
        t0 = time.time()
        while not srv.started:
            assert time.time() - t0 < 30
            time.sleep(0.05)
        res = terminal.evaluate(client.chat_policy(f"http://127.0.0.1:{port}"), tasks, max_turns=4, sandbox="local")
        assert res["solved"] == 2
        assert json.loads(res["episodes"][0].messages[1]["content"])["commands"]
    finally:
        srv.should_exit = True
        th.join(timeout=10)


def test_logits_match_transformers_qwen3(tmp_path):
    """Our Qwen3 forward (learned q/k norms, GQA, Llama-3 RoPE scaling, SwiGLU) against transformers'
    Qwen3ForCausalLM loaded from our export."""
    import warnings

    from transformers import Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=300, hidden_dim=64, intermediate_dim=128, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=32, rope_theta=500000.0,
                      rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 64},
                      norm_eps=1e-5, max_seq_len=256)
    m = Qwen3Model(cfg).init_weights(2)
    d = export_hf(m, str(tmp_path / "hf"), dtype=torch.float32)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        hf = Qwen3ForCausalLM.from_pretrained(d, torch_dtype=torch.float32).eval()
    tok = torch.randint(0, 300, (2, 40), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = hf(input_ids=tok).logits
        got = m.forward_reference(tok)
    assert torch.allclose(got.float(), want.float(), atol=2e-4, rtol=2e-4), (got - want).abs().max()
