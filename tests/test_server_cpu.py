"""OpenAI-compatible server over the continuous-batching engine (CPU, in-process client)."""
import json

import torch
from fastapi.testclient import TestClient

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.data import ByteTokenizer
from complexity_framework_b200.inference import GenerationConfig, InferenceEngine
from complexity_framework_b200.inference.server import ServingEngine, create_app


def _setup():
    tok = ByteTokenizer()
    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=tok.vocab_size,
                                    intermediate_size=64, shared_intermediate_size=128,
                                    num_experts=4, top_k=2, routing_strategy="modulo_cyclic",
                                    max_position_embeddings=256)).eval()
    return m, tok


def test_completions_match_engine_and_stream():
    m, tok = _setup()
    srv = ServingEngine(m, tok)
    try:
        c = TestClient(create_app(srv))
        r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 6}).json()
        ref = InferenceEngine(m).generate_tokens([tok.encode("hello")],
                                                 GenerationConfig(max_new_tokens=6))[0]
        assert r["choices"][0]["token_ids"] == ref
        assert r["usage"]["completion_tokens"] == 6
        with c.stream("POST", "/v1/chat/completions",
                      json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4,
                            "stream": True}) as s:
            lines = [l for l in s.iter_lines() if l.startswith("data: ")]
        assert lines[-1] == "data: [DONE]" and len(lines) == 5
        assert json.loads(lines[0][6:])["object"] == "chat.completion.chunk"
        assert c.get("/health").json()["status"] == "ok"
        assert "cfb_requests 2" in c.get("/metrics").text
    finally:
        srv.close()


def test_concurrent_requests_batch_together():
    import threading

    m, tok = _setup()
    srv = ServingEngine(m, tok)
    try:
        c = TestClient(create_app(srv))
        res = {}

        def go(i):
            res[i] = c.post("/v1/completions", json={"prompt": [1 + i, 2, 3],
                                                     "max_tokens": 5}).json()
        ts = [threading.Thread(target=go, args=(i,)) for i in range(4)]
        [t.start() for t in ts]
        [t.join() for t in ts]
        assert all(len(res[i]["choices"][0]["token_ids"]) == 5 for i in range(4))
    finally:
        srv.close()
