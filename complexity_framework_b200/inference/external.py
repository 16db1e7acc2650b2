"""OpenAI-compatible external backends (vLLM, SGLang, this framework's server).

Counterpart of complexity/inference/external.py:21-130: generation
parameters as an OpenAI payload, a standard-library HTTP client for
``/v1/completions`` and ``/v1/chat/completions``, and a factory that
defaults the base URL per backend.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional
from urllib.error import HTTPError, URLError
from urllib.request import Request, urlopen

DEFAULT_URLS = {"vllm": "http://127.0.0.1:8000", "sglang": "http://127.0.0.1:30000",
                "complexity": "http://127.0.0.1:8000", "openai": "http://127.0.0.1:8000"}


@dataclass
class ExternalGenerationConfig:
    max_tokens: int = 256
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: Optional[int] = None
    stop: Optional[List[str]] = None
    extra: Dict[str, Any] = field(default_factory=dict)

    def to_payload(self) -> Dict[str, Any]:
        p: Dict[str, Any] = {"max_tokens": self.max_tokens, "temperature": self.temperature,
                             "top_p": self.top_p}
        if self.top_k is not None:
            p["top_k"] = self.top_k
        if self.stop:
            p["stop"] = list(self.stop)
        p.update(self.extra)
        return p


class OpenAICompatibleBackend:
    def __init__(self, *, backend: str, base_url: str, model: str, api_key: Optional[str] = None,
                 timeout: float = 60.0):
        self.backend, self.base_url = backend, base_url.rstrip("/")
        self.model, self.api_key, self.timeout = model, api_key, timeout

    def _post_json(self, path: str, payload: Dict[str, Any]) -> Dict[str, Any]:
        headers = {"Content-Type": "application/json"}
        if self.api_key:
            headers["Authorization"] = f"Bearer {self.api_key}"
        req = Request(self.base_url + path, data=json.dumps(payload).encode(), headers=headers,
                      method="POST")
        try:
            with urlopen(req, timeout=self.timeout) as r:
                return json.loads(r.read().decode("utf-8"))
        except HTTPError as exc:
            body = exc.read().decode("utf-8", errors="replace")
            raise RuntimeError(f"{self.backend} request failed with HTTP {exc.code}: {body}") \
                from exc
        except URLError as exc:
            raise RuntimeError(f"{self.backend} server unreachable at {self.base_url}: "
                               f"{exc.reason}") from exc

    def complete(self, prompt: str, config: Optional[ExternalGenerationConfig] = None) -> str:
        cfg = config or ExternalGenerationConfig()
        out = self._post_json("/v1/completions", {"model": self.model, "prompt": prompt,
                                                  **cfg.to_payload()})
        try:
            return out["choices"][0]["text"]
        except (KeyError, IndexError, TypeError) as exc:
            raise RuntimeError(f"Invalid {self.backend} completion response: {out!r}") from exc

    def chat(self, messages: List[Dict[str, str]],
             config: Optional[ExternalGenerationConfig] = None) -> str:
        cfg = config or ExternalGenerationConfig()
        out = self._post_json("/v1/chat/completions", {"model": self.model, "messages": messages,
                                                       **cfg.to_payload()})
        try:
            return out["choices"][0]["message"]["content"]
        except (KeyError, IndexError, TypeError) as exc:
            raise RuntimeError(f"Invalid {self.backend} chat response: {out!r}") from exc


def create_external_backend(backend: str = "vllm", *, model: str,
                            base_url: Optional[str] = None, api_key: Optional[str] = None,
                            timeout: float = 60.0) -> OpenAICompatibleBackend:
    b = backend.lower()
    if b not in DEFAULT_URLS:
        raise ValueError(f"unknown external backend {backend!r}; choose from {sorted(DEFAULT_URLS)}")
    return OpenAICompatibleBackend(backend=b, base_url=base_url or DEFAULT_URLS[b], model=model,
                                   api_key=api_key, timeout=timeout)
