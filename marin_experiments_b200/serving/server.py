"""HTTP serving (tunix-delphi-rl/serving/serve.py:81-135,992-1068): ``GET /health``,
``POST /generate`` (``prompt`` or ``prompts``), an OpenAI-style ``POST /v1/completions``, ``POST
/calc`` (the calculator tool loop of the tool-calling RL task served live: the model writes
``CALC(a * b)``, the server multiplies and answers ``Tool result: N``, until the model gives a
final answer; the transcript, the calls and the answer come back) and a self-contained dashboard
page at ``/`` (no external scripts) that posts to those endpoints.

The engine's KV cache is shared state, and FastAPI runs synchronous endpoints on a thread pool,
so every generation runs under one lock: requests are served one after another (a batch of
prompts in one request still decodes together).

Run: ``python -m marin_experiments_b200.serving.server --model-dir <hf snapshot> [--port 8000]``
(``--random-tiny`` serves a small random-init model for smoke tests).
"""

from __future__ import annotations

import argparse
from typing import List, Optional

from pydantic import BaseModel


class GenerateRequest(BaseModel):
    prompt: Optional[str] = None
    prompts: Optional[List[str]] = None
    max_tokens: Optional[int] = None
    temperature: float = 0.8
    top_p: float = 1.0
    seed: int = 0
    stop: Optional[List[str]] = None

    def resolve_prompts(self) -> tuple[list[str], bool]:
        if self.prompts is not None and self.prompt is not None:
            raise ValueError("Pass exactly one of `prompt` or `prompts`.")
        if self.prompts is not None:
            if not self.prompts:
                raise ValueError("`prompts` must be non-empty.")
            return list(self.prompts), True
        if self.prompt is not None:
            return [self.prompt], False
        raise ValueError("Pass `prompt` (str) or `prompts` (list[str]).")


class GenerateResponse(BaseModel):
    text: Optional[str] = None
    texts: Optional[List[str]] = None


class CalcRequest(BaseModel):
    question: str  # e.g. "12 * 34 * 56" or "Q: 12 * 34 * 56"
    max_turns: int = 0  # 0: one more than the number of multiplications
    temperature: float = 0.0
    seed: int = 0


class CompletionRequest(BaseModel):
    prompt: str
    max_tokens: int = 256
    temperature: float = 0.8
    top_p: float = 1.0
    seed: int = 0
    stop: Optional[List[str]] = None


_DASHBOARD = """<!doctype html><html><head><meta charset="utf-8"><title>{name}</title>
<style>body{{font-family:sans-serif;max-width:52em;margin:2em auto}}textarea{{width:100%;height:8em}}
pre{{background:#f4f4f4;padding:1em;white-space:pre-wrap}}</style></head><body>
<h2>{name}</h2>
<h3>Generate</h3><textarea id="p">def fib(n):</textarea><br>
max tokens <input id="m" value="64" size="4"> temperature <input id="t" value="0" size="4">
<button onclick="gen()">generate</button><pre id="o"></pre>
<h3>Calculator agent</h3><input id="q" value="12 * 34 * 56" size="30"> <button onclick="calc()">solve</button>
<pre id="c"></pre>
<script>
async function post(url, body) {{
  const r = await fetch(url, {{method: "POST", headers: {{"content-type": "application/json"}},
                              body: JSON.stringify(body)}});
  return r.json();
}}
async function gen() {{
  const j = await post("/generate", {{prompt: document.getElementById("p").value,
    max_tokens: parseInt(document.getElementById("m").value),
    temperature: parseFloat(document.getElementById("t").value)}});
  document.getElementById("o").textContent = j.text !== undefined ? j.text : JSON.stringify(j);
}}
async function calc() {{
  const j = await post("/calc", {{question: document.getElementById("q").value}});
  document.getElementById("c").textContent = j.transcript !== undefined ?
    j.transcript + "\\n\\nanswer: " + j.answer + " (correct: " + j.correct + ")" : JSON.stringify(j);
}}
</script></body></html>"""


def build_app(engine, model_name: str = "qwen3"):
    import html
    import threading

    from fastapi import FastAPI, HTTPException
    from fastapi.responses import HTMLResponse

    app = FastAPI(title="marin_experiments_b200 serving", version="0.1.0")
    lock = threading.Lock()

    def run(prompts, **kw):
        with lock:
            try:
                return engine.generate(prompts, **kw)
            except ValueError as exc:  # e.g. prompt + max_tokens beyond the KV cache: the request's fault
                raise HTTPException(status_code=400, detail=str(exc)) from exc

    @app.get("/", response_class=HTMLResponse)
    @app.get("/dashboard", response_class=HTMLResponse)
    def dashboard() -> str:
        return _DASHBOARD.format(name=html.escape(model_name))

    @app.get("/health")
    def health() -> dict:
        return {"ok": bool(engine.ready), "model": model_name}

    @app.post("/generate", response_model=GenerateResponse)
    def generate(req: GenerateRequest) -> GenerateResponse:
        if not engine.ready:
            raise HTTPException(status_code=503, detail="model loading")
        try:
            prompts, batched = req.resolve_prompts()
        except ValueError as exc:
            raise HTTPException(status_code=400, detail=str(exc)) from exc
        texts = run(prompts, max_tokens=req.max_tokens, temperature=req.temperature, top_p=req.top_p, seed=req.seed,
                    stop=req.stop)
        return GenerateResponse(texts=texts) if batched else GenerateResponse(text=texts[0])

    @app.post("/v1/completions")
    def completions(req: CompletionRequest) -> dict:
        if not engine.ready:
            raise HTTPException(status_code=503, detail="model loading")
        texts = run([req.prompt], max_tokens=req.max_tokens, temperature=req.temperature, top_p=req.top_p,
                    seed=req.seed, stop=req.stop)
        return {"object": "text_completion", "model": model_name,
                "choices": [{"index": 0, "text": texts[0], "finish_reason": "stop"}]}

    @app.post("/calc")
    def calc(req: CalcRequest) -> dict:
        from ..rl import tools

        if not engine.ready:
            raise HTTPException(status_code=503, detail="model loading")
        q = req.question.strip()
        q = q[2:].strip() if q.startswith("Q:") else q
        try:
            ops = tuple(int(v) for v in q.split("*"))
        except ValueError:
            raise HTTPException(status_code=400, detail="question must be integers joined by '*'") from None
        if not 2 <= len(ops) <= 16 or not 0 <= req.max_turns <= 17:
            raise HTTPException(status_code=400, detail="question needs 2 to 16 factors; max_turns 0 to 17")
        prod = 1
        for v in ops:
            prod *= v
        task = tools.ChainTask("Q: " + " * ".join(map(str, ops)), ops, str(prod))
        env = tools.rollout(lambda text: run([text], max_tokens=32, temperature=req.temperature, seed=req.seed,
                                             stop=["\n"])[0], task, req.max_turns)
        return {"transcript": env.render()[len(env.system) + 1:].rstrip("\n"), "answer": env.final_answer,
                "calls": env.calls, "correct": env.reward() >= 1.0, "reward": tools.total_reward(env)}

    app.state.engine = engine
    return app


def tiny_engine(device="cpu"):
    """A small random-init Qwen3 with the byte tokenizer (tests and smoke runs)."""
    from ..data.tokenize import ByteTokenizer
    from ..models.qwen3 import Qwen3Config, Qwen3Model
    from .engine import Engine

    cfg = Qwen3Config(vocab_size=512, hidden_dim=128, intermediate_dim=256, num_layers=2, num_heads=2, num_kv_heads=1,
                      head_dim=64, rope_theta=10000.0, max_seq_len=256)
    model = Qwen3Model(cfg).init_weights(0).to(device)
    return Engine(model, ByteTokenizer(), device=device, max_batch=4, max_len=256)


def main(argv=None):
    import torch
    import uvicorn

    ap = argparse.ArgumentParser()
    ap.add_argument("--model-dir", default=None)
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--random-tiny", action="store_true")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-batch", type=int, default=8)
    args = ap.parse_args(argv)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    if args.random_tiny or not args.model_dir:
        engine, name = tiny_engine(dev), "random-tiny"
    else:
        from ..data.tokenize import load_tokenizer
        from ..models.qwen3 import load_hf
        from .engine import Engine

        model = load_hf(args.model_dir, device=dev)
        engine = Engine(model, load_tokenizer(args.tokenizer or args.model_dir), device=dev, max_batch=args.max_batch)
        name = args.model_dir
    uvicorn.run(build_app(engine, name), host=args.host, port=args.port)


if __name__ == "__main__":
    main()
