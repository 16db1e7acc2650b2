"""Reference-API KV caches, external backend client and self-speculative decoding."""
import json
import threading
from http.server import BaseHTTPRequestHandler, HTTPServer

import pytest
import torch

from complexity_framework_b200.inference.external import (ExternalGenerationConfig,
                                                          create_external_backend)
from complexity_framework_b200.inference.kv_cache import CacheConfig, PagedKVCache, create_cache


def test_paged_kv_cache_update_gathers_sequence():
    c = PagedKVCache(num_layers=2, num_heads=2, head_dim=4, page_size=4, num_pages=8)
    c.allocate_sequence(7)
    ks = []
    for t in range(6):
        k = torch.full((1, 2, 1, 4), float(t))
        K, V = c.update(7, 1, k, -k)
        c.advance(7)
        ks.append(float(t))
        assert K.shape == (1, 2, t + 1, 4) and K[0, 0, :, 0].tolist() == ks
    assert c.get_seq_len(7) == 6 and c.memory_usage()["used_pages"] == 2
    c.free_sequence(7)
    assert c.memory_usage()["used_pages"] == 0
    std = create_cache(CacheConfig(2, 2, 4, 16, dtype=torch.float32), "standard")
    std.update(0, torch.ones(1, 2, 3, 4), torch.ones(1, 2, 3, 4))
    assert std.memory_usage() > 0
    assert isinstance(create_cache(CacheConfig(2, 2, 4, 16), "paged", num_pages=4), PagedKVCache)
    with pytest.raises(ValueError):
        create_cache(CacheConfig(2, 2, 4, 16), "ring")


def test_external_backend_against_local_server():
    seen = {}

    class H(BaseHTTPRequestHandler):
        def do_POST(self):
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            seen[self.path] = (body, self.headers.get("Authorization"))
            out = ({"choices": [{"text": "done"}]} if self.path == "/v1/completions" else
                   {"choices": [{"message": {"content": "hello"}}]})
            data = json.dumps(out).encode()
            self.send_response(200)
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def log_message(self, *a):
            pass

    srv = HTTPServer(("127.0.0.1", 0), H)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        b = create_external_backend("vllm", model="m", api_key="k",
                                    base_url=f"http://127.0.0.1:{srv.server_port}")
        assert b.complete("x", ExternalGenerationConfig(max_tokens=3, top_k=5)) == "done"
        assert b.chat([{"role": "user", "content": "hi"}]) == "hello"
        body, auth = seen["/v1/completions"]
        assert body["max_tokens"] == 3 and body["top_k"] == 5 and auth == "Bearer k"
    finally:
        srv.shutdown()
    with pytest.raises(ValueError):
        create_external_backend("tgi", model="m")


def test_self_speculative_decoder_matches_greedy():
    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.inference.decoding import (SelfSpeculativeDecoder,
                                                              SpeculativeConfig)

    torch.manual_seed(0)
    m = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=3, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=97, intermediate_size=64,
                                    shared_intermediate_size=128, num_experts=2, top_k=2,
                                    max_position_embeddings=128)).eval()
    ids = torch.randint(0, 97, (1, 6))
    dec = SelfSpeculativeDecoder(m, exit_layer=1, config=SpeculativeConfig(3, temperature=1.0))
    out = dec.generate(ids, max_new_tokens=8)
    ref = ids.clone()
    with torch.no_grad():
        for _ in range(8):
            nxt = m(ref)["logits"][:, -1].argmax(-1, keepdim=True)
            ref = torch.cat([ref, nxt], 1)
    assert torch.equal(out, ref)
