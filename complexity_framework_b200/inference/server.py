"""OpenAI-compatible HTTP serving and an external-backend client.

Counterparts: ``complexity serve start`` / ``openai-proxy``
(complexity/cli/commands/serve.py), the batcher-backed serving of
complexity/inference/engine.py and the OpenAI-compatible client of
complexity/inference/external.py.

``ServingEngine`` owns an ``InferenceEngine`` and drives it from one
background thread: requests from any number of HTTP handlers join the
continuously-batched decode between steps, and each request's new tokens are
pushed to its own queue (streaming responses read them as they arrive).
``create_app`` builds the FastAPI app: ``/v1/completions``,
``/v1/chat/completions`` (both with ``stream``), ``/v1/models``, ``/health``
and Prometheus ``/metrics``.
"""
from __future__ import annotations

import json
import queue
import threading
import time
import uuid
from typing import Any, Dict, Iterator, List, Optional

import torch

from .engine import GenerationConfig, InferenceConfig, InferenceEngine

_DONE = object()


class ServingEngine:
    def __init__(self, model, tokenizer, config: Optional[InferenceConfig] = None,
                 model_name: str = "complexity"):
        self.engine = InferenceEngine(model, config)
        self.tok = tokenizer
        self.model_name = model_name
        self._lock = threading.Lock()
        self._wake = threading.Event()
        self._queues: Dict[int, "queue.Queue"] = {}
        self._sent: Dict[int, int] = {}
        self._stop = False
        self.metrics = {"requests": 0, "tokens_out": 0, "tokens_in": 0}
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()

    def _loop(self) -> None:
        while not self._stop:
            with self._lock:
                pending = self.engine.has_pending()
            if not pending:
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            with self._lock:
                finished = set(self.engine.step())
                for rid, q in list(self._queues.items()):
                    r = self.engine.requests.get(rid)
                    if r is None:
                        continue
                    sent = self._sent[rid]
                    for t in r.output[sent:]:
                        q.put(t)
                    self._sent[rid] = len(r.output)
                    if rid in finished:
                        q.put(_DONE)
                        self.metrics["tokens_out"] += len(r.output)
                        self.engine.requests.pop(rid, None)
                        del self._queues[rid]
                        del self._sent[rid]

    def submit(self, prompt_ids: List[int], gen: GenerationConfig) -> "queue.Queue":
        q: "queue.Queue" = queue.Queue()
        with self._lock:
            rid = self.engine.add_request(prompt_ids, gen)
            self._queues[rid] = q
            self._sent[rid] = 0
            self.metrics["requests"] += 1
            self.metrics["tokens_in"] += len(prompt_ids)
        self._wake.set()
        return q

    @staticmethod
    def drain(q: "queue.Queue", timeout: float = 600.0) -> Iterator[int]:
        while True:
            item = q.get(timeout=timeout)
            if item is _DONE:
                return
            yield item

    def close(self) -> None:
        self._stop = True
        self._wake.set()
        self._thread.join(timeout=5)


def _gen_config(body: Dict[str, Any], eos: Optional[int]) -> GenerationConfig:
    temp = float(body.get("temperature", 0.0) or 0.0)
    return GenerationConfig(max_new_tokens=int(body.get("max_tokens", 64)),
                            do_sample=temp > 0, temperature=temp if temp > 0 else 1.0,
                            top_p=float(body.get("top_p", 1.0) or 1.0),
                            top_k=int(body.get("top_k", 0) or 0),
                            repetition_penalty=float(body.get("repetition_penalty", 1.0) or 1.0),
                            eos_token_id=eos, seed=body.get("seed"))


def create_app(serving: ServingEngine):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse

    app = FastAPI(title="complexity_framework_b200 server")
    tok = serving.tok

    def _prompt_ids(body) -> List[int]:
        p = body.get("prompt")
        if isinstance(p, list) and all(isinstance(x, int) for x in p):
            return p
        if isinstance(p, str):
            return tok.encode(p)
        raise HTTPException(400, "prompt must be a string or a list of token ids")

    def _chat_ids(body) -> List[int]:
        from ..data.tokenization import ChatTemplate

        msgs = body.get("messages")
        if not msgs:
            raise HTTPException(400, "messages required")
        fmt = body.get("chat_format", "complexity")
        return tok.encode(ChatTemplate(fmt).apply(msgs, add_generation_prompt=True))

    def _respond(ids, body, chat: bool):
        gen = _gen_config(body, tok.eos_token_id)
        q = serving.submit(ids, gen)
        rid = f"cmpl-{uuid.uuid4().hex[:12]}"
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        if body.get("stream"):
            def events():
                for t in ServingEngine.drain(q):
                    piece = tok.decode([t])
                    delta = ({"delta": {"content": piece}, "index": 0} if chat else
                             {"text": piece, "index": 0})
                    yield "data: " + json.dumps({"id": rid, "object": obj + ".chunk",
                                                 "created": created, "model": serving.model_name,
                                                 "choices": [delta]}) + "\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(events(), media_type="text/event-stream")
        out = list(ServingEngine.drain(q))
        text = tok.decode(out)
        choice = ({"message": {"role": "assistant", "content": text}, "index": 0,
                   "finish_reason": "stop"} if chat else
                  {"text": text, "index": 0, "finish_reason": "stop", "token_ids": out})
        return {"id": rid, "object": obj, "created": created, "model": serving.model_name,
                "choices": [choice],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                          "total_tokens": len(ids) + len(out)}}

    @app.post("/v1/completions")
    def completions(body: Dict[str, Any]):
        return _respond(_prompt_ids(body), body, chat=False)

    @app.post("/v1/chat/completions")
    def chat(body: Dict[str, Any]):
        return _respond(_chat_ids(body), body, chat=True)

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": serving.model_name, "object": "model"}]}

    @app.get("/health")
    def health():
        return {"status": "ok"}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        st = dict(serving.metrics, **serving.engine.get_serving_stats())
        lines = []
        for k, v in st.items():
            if isinstance(v, (int, float)):
                lines.append(f"cfb_{k} {v}")
        return "\n".join(lines) + "\n"

    return app


def serve(model, tokenizer, host: str = "127.0.0.1", port: int = 8000,
          config: Optional[InferenceConfig] = None, model_name: str = "complexity") -> None:
    import uvicorn

    serving = ServingEngine(model, tokenizer, config, model_name)
    try:
        uvicorn.run(create_app(serving), host=host, port=port)
    finally:
        serving.close()


class ExternalBackend:
    """Client of an OpenAI-compatible server (this one, vLLM, SGLang ...)."""

    def __init__(self, base_url: str, model: str = "complexity", api_key: Optional[str] = None,
                 backend: str = "openai", timeout: float = 120.0):
        self.base_url = base_url.rstrip("/")
        self.model, self.api_key, self.backend, self.timeout = model, api_key, backend, timeout

    def _post(self, path: str, body: Dict) -> Dict:
        import requests

        h = {"Authorization": f"Bearer {self.api_key}"} if self.api_key else {}
        r = requests.post(self.base_url + path, json=body, headers=h, timeout=self.timeout)
        r.raise_for_status()
        return r.json()

    def complete(self, prompt: str, **kw) -> str:
        return self._post("/v1/completions", {"model": self.model, "prompt": prompt, **kw})[
            "choices"][0]["text"]

    def chat(self, messages: List[Dict[str, str]], **kw) -> str:
        return self._post("/v1/chat/completions", {"model": self.model, "messages": messages,
                                                   **kw})["choices"][0]["message"]["content"]
