"""Continuous batching front end (API of complexity/inference/batching.py:25-416).

``ContinuousBatcher`` keeps the reference's request/status/statistics API but
runs on the paged engine: requests decode against their KV pages instead of
re-running the full prefix every step (the reference batcher recomputes the
whole padded batch per token).
"""
from __future__ import annotations

import threading
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional

import torch

from .engine import GenerationConfig, InferenceConfig, InferenceEngine


class RequestStatus(Enum):
    PENDING = "pending"
    RUNNING = "running"
    COMPLETED = "completed"
    FAILED = "failed"


@dataclass
class Request:
    input_ids: Any
    request_id: str = ""
    max_tokens: int = 100
    temperature: float = 1.0
    top_k: Optional[int] = None
    top_p: Optional[float] = None
    stop_tokens: Optional[List[int]] = None
    output_ids: List[int] = field(default_factory=list)
    status: RequestStatus = RequestStatus.PENDING
    arrival_time: float = 0.0
    start_time: float = 0.0
    end_time: float = 0.0
    position: int = 0
    tokens_generated: int = 0

    def __post_init__(self):
        if not self.request_id:
            self.request_id = f"req-{int(time.time() * 1_000_000)}-{id(self) & 0xffff}"


@dataclass
class BatchConfig:
    max_batch_size: int = 32
    max_sequence_length: int = 2048
    max_tokens_per_batch: Optional[int] = None
    prefill_chunk_size: int = 512
    dynamic_batching: bool = True
    timeout_seconds: float = 60.0


class ContinuousBatcher:
    def __init__(self, model, config: Optional[BatchConfig] = None, page_size: int = 16):
        self.config = config or BatchConfig()
        icfg = InferenceConfig(max_cache_length=self.config.max_sequence_length,
                               max_batch_size=self.config.max_batch_size, page_size=page_size,
                               max_tokens_per_step=self.config.max_tokens_per_batch or 8192,
                               prefill_chunk_size=self.config.prefill_chunk_size)
        self.engine = InferenceEngine(model, icfg)
        self.requests: Dict[str, Request] = {}
        self._eng_ids: Dict[int, str] = {}
        self.completed: List[Request] = []

    def add_request(self, request: Request) -> str:
        ids = request.input_ids
        ids = ids.reshape(-1).tolist() if isinstance(ids, torch.Tensor) else list(ids)
        sampling = request.temperature > 0 and (request.top_k or request.top_p)
        gen = GenerationConfig(max_new_tokens=request.max_tokens, do_sample=bool(sampling),
                               temperature=request.temperature, top_k=request.top_k or 0,
                               top_p=request.top_p if request.top_p is not None else 1.0,
                               stop_sequences=[[t] for t in (request.stop_tokens or [])])
        request.arrival_time = time.perf_counter()
        eid = self.engine.add_request(ids, gen)
        self._eng_ids[eid] = request.request_id
        self.requests[request.request_id] = request
        return request.request_id

    def has_pending(self) -> bool:
        return self.engine.has_pending()

    def step(self) -> List[Request]:
        """Advance every active request by one engine step; returns newly completed ones."""
        done_ids = self.engine.step()
        for eid in list(self.engine.running):
            req = self.requests[self._eng_ids[eid]]
            if req.status is RequestStatus.PENDING:
                req.status = RequestStatus.RUNNING
                req.start_time = time.perf_counter()
            req.output_ids = list(self.engine.requests[eid].output)
            req.tokens_generated = len(req.output_ids)
        finished = []
        for eid in done_ids:
            req = self.requests[self._eng_ids.pop(eid)]
            req.output_ids = list(self.engine.requests.pop(eid).output)
            req.tokens_generated = len(req.output_ids)
            req.status = RequestStatus.COMPLETED
            req.end_time = time.perf_counter()
            finished.append(req)
            self.completed.append(req)
        return finished

    def run_until_complete(self) -> List[Request]:
        while self.has_pending():
            self.step()
        return self.completed

    def get_request(self, request_id: str) -> Optional[Request]:
        return self.requests.get(request_id)

    def cancel_request(self, request_id: str) -> bool:
        for eid, rid in list(self._eng_ids.items()):
            if rid == request_id:
                r = self.engine.requests[eid]
                if eid in self.engine.waiting:
                    self.engine.waiting.remove(eid)
                if eid in self.engine.running:
                    self.engine.running.remove(eid)
                if eid in self.engine.pool.pages:
                    self.engine.pool.free_sequence(eid)
                r.done = True
                self.requests[request_id].status = RequestStatus.FAILED
                self._eng_ids.pop(eid)
                return True
        return False

    def get_statistics(self) -> Dict[str, Any]:
        lat = [r.end_time - r.arrival_time for r in self.completed]
        toks = sum(r.tokens_generated for r in self.completed)
        return {"completed": len(self.completed), "active": len(self._eng_ids),
                "total_tokens": toks,
                "mean_latency_s": sum(lat) / len(lat) if lat else 0.0,
                **self.engine.get_serving_stats()}


class AsyncBatcher(ContinuousBatcher):
    """Background-thread driver of the batcher."""

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self._lock = threading.Lock()
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()

    def start(self) -> None:
        self._stop.clear()
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=10)

    def _loop(self) -> None:
        while not self._stop.is_set():
            with self._lock:
                busy = self.has_pending()
                if busy:
                    self.step()
            if not busy:
                time.sleep(0.001)

    def add_request_async(self, request: Request) -> str:
        with self._lock:
            return self.add_request(request)
