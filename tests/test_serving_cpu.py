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
