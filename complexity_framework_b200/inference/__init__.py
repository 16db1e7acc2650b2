"""Inference: paged KV cache, continuous-batching engine, sampling."""
from .batching import AsyncBatcher, BatchConfig, ContinuousBatcher, Request, RequestStatus
from .engine import (DecodingStrategy, GenerationConfig, InferenceConfig, InferenceEngine,
                     forward_paged, sample_next)
from .decoding import (LayerSkipDraft, SlidingWindowCache, SpeculativeDecoder, SpeculativeStats,
                       beam_search, paged_logits)
from .paged import KVCache, OutOfPages, PagedBatch, PagePool, SeqChunk
from . import chat_template  # noqa: F401  (template contract: inference.chat_template)

PagedKVCache = PagePool

__all__ = ["AsyncBatcher", "BatchConfig", "ContinuousBatcher", "DecodingStrategy",
           "GenerationConfig", "InferenceConfig", "InferenceEngine", "KVCache", "OutOfPages",
           "PagedBatch", "PagedKVCache", "PagePool", "Request", "RequestStatus", "SeqChunk",
           "forward_paged", "sample_next", "LayerSkipDraft", "SlidingWindowCache",
           "SpeculativeDecoder", "SpeculativeStats", "beam_search", "paged_logits"]
