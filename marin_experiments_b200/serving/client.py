"""Client of the serving API (tunix-delphi-rl/serving/query.py:1-187): ``health``, ``generate`` (one
prompt or a batch through ``POST /generate``) and ``complete`` (``POST /v1/completions``), over
plain HTTP with a timeout, plus a command line. The reference resolves its endpoint through its
cluster's proxy; here the caller passes the server's base URL (``--url`` or ``MXK_SERVE_URL``).

``chat_policy`` / ``text_policy`` wrap a served model as the policy callables the RL environments
and agent evaluations take.

``python -m marin_experiments_b200.serving.client --url http://127.0.0.1:8000 --prompt "def f():"
--max-tokens 64 --temperature 0``
"""

from __future__ import annotations

import json
import os
import sys
import urllib.error
import urllib.request


class ServingError(RuntimeError):
    pass


def _post(url: str, path: str, body: dict, timeout_s: float) -> dict:
    rq = urllib.request.Request(url.rstrip("/") + path, data=json.dumps(body).encode(), method="POST",
                                headers={"content-type": "application/json"})
    try:
        with urllib.request.urlopen(rq, timeout=timeout_s) as r:
            return json.loads(r.read())
    except urllib.error.HTTPError as e:
        raise ServingError(f"{path}: HTTP {e.code}: {e.read().decode(errors='replace')}") from None


def health(url: str, timeout_s: float = 10.0) -> dict:
    with urllib.request.urlopen(url.rstrip("/") + "/health", timeout=timeout_s) as r:
        return json.loads(r.read())


def generate(url: str, prompt: str | list[str], *, max_tokens: int | None = None, temperature: float = 0.8,
             top_p: float = 1.0, seed: int = 0, stop: list[str] | None = None,
             timeout_s: float = 300.0) -> str | list[str]:
    """The continuation of ``prompt`` (a list of prompts gives a list of continuations)."""
    body = {"max_tokens": max_tokens, "temperature": temperature, "top_p": top_p, "seed": seed, "stop": stop}
    batched = isinstance(prompt, list)
    body["prompts" if batched else "prompt"] = prompt
    out = _post(url, "/generate", body, timeout_s)
    return out["texts"] if batched else out["text"]


def complete(url: str, prompt: str, *, max_tokens: int = 256, temperature: float = 0.8, top_p: float = 1.0,
             seed: int = 0, stop: list[str] | None = None, timeout_s: float = 300.0) -> str:
    out = _post(url, "/v1/completions", {"prompt": prompt, "max_tokens": max_tokens, "temperature": temperature,
                                         "top_p": top_p, "seed": seed, "stop": stop}, timeout_s)
    return out["choices"][0]["text"]


def chat_policy(url: str, *, max_tokens: int = 512, temperature: float = 0.0, timeout_s: float = 300.0):
    """A served model as an agent policy (openthoughts-agent/eval/model_serving.py): ``messages ->
    reply``, rendering the conversation as ChatML with an open assistant turn and stopping at the end
    marker -- the ``model_fn`` that ``rl.terminal.evaluate`` and ``rl.agent.run_episode`` take."""
    from ..data.chat import IM_END, render_chatml

    def policy(messages: list[dict]) -> str:
        text = generate(url, render_chatml(messages, add_generation_prompt=True), max_tokens=max_tokens,
                        temperature=temperature, stop=[IM_END], timeout_s=timeout_s)
        return text.split(IM_END, 1)[0]

    return policy


def text_policy(url: str, *, max_tokens: int = 64, temperature: float = 0.0, stop: list[str] | None = None,
                timeout_s: float = 300.0):
    """A served model as a raw-text policy (``text -> continuation``), for the few-shot environments."""

    def policy(text: str) -> str:
        return generate(url, text, max_tokens=max_tokens, temperature=temperature, stop=stop, timeout_s=timeout_s)

    return policy


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(prog="python -m marin_experiments_b200.serving.client")
    ap.add_argument("--url", default=os.environ.get("MXK_SERVE_URL", "http://127.0.0.1:8000"))
    ap.add_argument("--prompt", action="append", required=True, help="repeat for a batch")
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-p", type=float, default=1.0)
    ap.add_argument("--stop", action="append", default=None)
    ap.add_argument("--timeout", type=float, default=300.0)
    a = ap.parse_args(argv)
    p = a.prompt if len(a.prompt) > 1 else a.prompt[0]
    out = generate(a.url, p, max_tokens=a.max_tokens, temperature=a.temperature, top_p=a.top_p, stop=a.stop,
                   timeout_s=a.timeout)
    for t in (out if isinstance(out, list) else [out]):
        print(t)
    return 0


if __name__ == "__main__":
    sys.exit(main())
