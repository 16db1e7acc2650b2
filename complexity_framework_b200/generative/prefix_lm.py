"""Prefix language modelling shared by the speech-to-text and image-text-to-text
models: modality tokens (already in the decoder's hidden size) are placed in
front of the text embeddings, the TR-Hash decoder runs over the whole
sequence, and the loss covers only the text positions.  Modality positions
route through the decoder's experts with one reserved route id.

Counterpart: the decoder halves of complexity/generative/audio/model.py and
vision_language/model.py.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class PrefixLM(nn.Module):
    def __init__(self, decoder, prefix_route_id: int = 0):
        super().__init__()
        self.decoder = decoder
        self.prefix_route_id = prefix_route_id

    def _run(self, prefix: torch.Tensor, input_ids: torch.Tensor) -> torch.Tensor:
        emb = self.decoder.embed_tokens(input_ids)
        x = torch.cat([prefix.to(emb.dtype), emb], 1)
        B, P = prefix.shape[:2]
        route = torch.cat([torch.full((B, P), self.prefix_route_id, dtype=torch.long,
                                      device=input_ids.device), input_ids], 1)
        out = self.decoder(inputs_embeds=x, routing_ids=route)
        return out["logits"][:, P:]

    def loss(self, prefix: torch.Tensor, input_ids: torch.Tensor,
             labels: Optional[torch.Tensor] = None, ignore_index: int = -100) -> torch.Tensor:
        logits = self._run(prefix, input_ids)
        tgt = (labels if labels is not None else input_ids)[:, 1:]
        return F.cross_entropy(logits[:, :-1].float().reshape(-1, logits.shape[-1]),
                               tgt.reshape(-1), ignore_index=ignore_index)

    @torch.no_grad()
    def generate(self, prefix: torch.Tensor, bos_ids: torch.Tensor, max_new_tokens: int = 32,
                 eos_id: Optional[int] = None, use_cache: bool = True) -> torch.Tensor:
        """Greedy decoding after the prefix; returns [B, T + new] token ids.  With
        ``use_cache`` the prefix and prompt run once and every new token is one
        decoder step over the key/value cache."""
        if not use_cache:
            ids = bos_ids
            for _ in range(max_new_tokens):
                nxt = self._run(prefix, ids)[:, -1].argmax(-1, keepdim=True)
                ids = torch.cat([ids, nxt], 1)
                if eos_id is not None and bool((nxt == eos_id).all()):
                    break
            return ids
        emb = self.decoder.embed_tokens(bos_ids)
        x = torch.cat([prefix.to(emb.dtype), emb], 1)
        B, P = prefix.shape[:2]
        route = torch.cat([torch.full((B, P), self.prefix_route_id, dtype=torch.long,
                                      device=bos_ids.device), bos_ids], 1)
        out = self.decoder(inputs_embeds=x, routing_ids=route, use_cache=True)
        ids = bos_ids
        for _ in range(max_new_tokens):
            nxt = out["logits"][:, -1].argmax(-1, keepdim=True)
            ids = torch.cat([ids, nxt], 1)
            if eos_id is not None and bool((nxt == eos_id).all()):
                break
            out = self.decoder(nxt, past_key_values=out["past_key_values"], use_cache=True)
        return ids


class TokenResampler(nn.Module):
    """A fixed number of learned queries cross-attend to a variable-length
    sequence (audio frames, image patches) and are projected to the decoder
    width: the modality's length no longer sets the prefix length."""

    def __init__(self, in_dim: int, out_dim: int, num_queries: int = 32, heads: int = 4):
        super().__init__()
        self.queries = nn.Parameter(torch.randn(1, num_queries, in_dim) * 0.02)
        self.norm = nn.LayerNorm(in_dim)
        self.attn = nn.MultiheadAttention(in_dim, heads, batch_first=True)
        self.mlp = nn.Sequential(nn.LayerNorm(in_dim), nn.Linear(in_dim, 4 * in_dim), nn.GELU(),
                                 nn.Linear(4 * in_dim, in_dim))
        self.proj = nn.Linear(in_dim, out_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        q = self.queries.expand(x.shape[0], -1, -1).to(x.dtype)
        kv = self.norm(x)
        q = q + self.attn(q, kv, kv, need_weights=False)[0]
        q = q + self.mlp(q)
        return self.proj(q)
