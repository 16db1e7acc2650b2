"""Beam search and speculative decoding over the paged KV cache.

Counterparts: the beam-search strategy of complexity/inference/engine.py
(``DecodingStrategy.BEAM_SEARCH``) and complexity/inference/speculative.py:26-469
(draft/verify speculative decoding, self-speculative early exit).

Both run on the same paged forward as the serving engine: a target model
verifies ``k`` drafted tokens in ONE ragged forward (a ``k+1``-token chunk
appended to its cache) and rejected tokens are rolled back by truncating the
sequence's page list; beams fork a parent's cache by copying its pages.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from .paged import PagedBatch, PagePool, SeqChunk


def _pool_for(model, num_seqs: int, max_len: int, page_size: int = 16) -> PagePool:
    mc = model.config
    p = next(model.parameters())
    pages = num_seqs * (-(-max_len // page_size) + 1)
    return PagePool(len(model.layers), mc.num_key_value_heads, mc.head_dim, pages, page_size,
                    dtype=p.dtype, device=p.device)


@torch.no_grad()
def paged_logits(model, pool: PagePool, chunks: Sequence[SeqChunk], toks: Sequence[int],
                 all_positions: bool = False) -> List[torch.Tensor]:
    """One ragged forward; per chunk the logits of its last token ``[V]`` (or of
    every token ``[len, V]`` with ``all_positions``)."""
    from .engine import forward_paged

    batch = PagedBatch(pool, chunks)
    dev = pool.device
    hidden = forward_paged(model, torch.tensor(list(toks), dtype=torch.long, device=dev), batch)
    batch.commit()
    cu = batch._cu_host
    if all_positions:
        lg = model.logits(hidden[None])[0].float()
        return [lg[cu[i]:cu[i + 1]] for i in range(len(chunks))]
    last = torch.tensor([c - 1 for c in cu[1:]], device=dev)
    lg = model.logits(hidden[last][None])[0].float()
    return [lg[i] for i in range(len(chunks))]


# ---------------------------------------------------------------- beam search
@dataclass
class BeamHypothesis:
    tokens: List[int]
    score: float

    def normalized(self, length_penalty: float) -> float:
        return self.score / (max(1, len(self.tokens)) ** length_penalty)


@torch.no_grad()
def beam_search(model, prompt: Sequence[int], num_beams: int = 4, max_new_tokens: int = 32,
                length_penalty: float = 1.0, eos_token_id: Optional[int] = None,
                page_size: int = 16) -> Dict:
    """Returns ``{"tokens": best continuation, "score": ..., "hypotheses": [...]}``."""
    prompt = list(prompt)
    pool = _pool_for(model, 2 * num_beams + 1, len(prompt) + max_new_tokens + 1, page_size)
    pool.allocate_sequence(0)
    lg = paged_logits(model, pool, [SeqChunk(0, 0, len(prompt))], prompt)[0]
    logp = torch.log_softmax(lg, -1)
    top = torch.topk(logp, num_beams)
    next_id = 1
    beams: List[Tuple[int, List[int], float]] = []
    for v, t in zip(top.values.tolist(), top.indices.tolist()):
        pool.fork_sequence(0, next_id)
        beams.append((next_id, [t], v))
        next_id += 1
    pool.free_sequence(0)
    done: List[BeamHypothesis] = []
    for step in range(max_new_tokens):
        alive = []
        for sid, toks, sc in beams:
            if eos_token_id is not None and toks[-1] == eos_token_id:
                done.append(BeamHypothesis(toks, sc))
                pool.free_sequence(sid)
            else:
                alive.append((sid, toks, sc))
        if not alive or step == max_new_tokens - 1:
            for sid, toks, sc in alive:
                done.append(BeamHypothesis(toks, sc))
                pool.free_sequence(sid)
            break
        chunks = [SeqChunk(sid, len(prompt) + len(toks) - 1, 1) for sid, toks, _ in alive]
        outs = paged_logits(model, pool, chunks, [toks[-1] for _, toks, _ in alive])
        cand = []
        for (sid, toks, sc), row in zip(alive, outs):
            lp = torch.log_softmax(row, -1)
            tv = torch.topk(lp, num_beams)
            for v, t in zip(tv.values.tolist(), tv.indices.tolist()):
                cand.append((sc + v, sid, toks, t))
        cand.sort(key=lambda c: -c[0])
        new_beams = []
        for score, parent, toks, t in cand[:num_beams]:
            pool.fork_sequence(parent, next_id)
            new_beams.append((next_id, toks + [t], score))
            next_id += 1
        for sid, _, _ in alive:
            pool.free_sequence(sid)
        beams = new_beams
    done.sort(key=lambda h: -h.normalized(length_penalty))
    best = done[0]
    return {"tokens": best.tokens, "score": best.normalized(length_penalty),
            "hypotheses": [(h.tokens, h.normalized(length_penalty)) for h in done]}


# --------------------------------------------------------- speculative decoding
class LayerSkipDraft(nn.Module):
    """Self-speculative draft: the first ``num_layers`` blocks of ``model`` plus
    its final norm and LM head (early exit), sharing the weights."""

    def __init__(self, model, num_layers: int):
        super().__init__()
        self.base = model
        self.layers = model.layers[:num_layers]
        self.config = model.config

    def parameters(self, recurse: bool = True):
        return self.base.parameters(recurse)

    def embed(self, ids):
        return self.base.embed(ids)

    @property
    def norm(self):
        return self.base.norm

    def logits(self, h):
        return self.base.logits(h)


@dataclass
class SpeculativeStats:
    drafted: int = 0
    accepted: int = 0
    target_forwards: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0


class SpeculativeDecoder:
    """Draft ``k`` tokens with ``draft``, verify them with ``target`` in one forward.

    Greedy (temperature 0) accepts the longest prefix on which the target's
    argmax agrees; with sampling, draft token x is accepted with probability
    min(1, p(x)/q(x)) and a rejection resamples from max(0, p - q), which
    leaves the output distribution equal to the target's.
    """

    def __init__(self, target, draft, num_draft_tokens: int = 4, page_size: int = 16):
        self.target, self.draft, self.k, self.page_size = target, draft, num_draft_tokens, page_size
        self.stats = SpeculativeStats()

    @torch.no_grad()
    def generate(self, prompt: Sequence[int], max_new_tokens: int = 32, temperature: float = 0.0,
                 eos_token_id: Optional[int] = None, seed: Optional[int] = None) -> List[int]:
        prompt = list(prompt)
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        cap = len(prompt) + max_new_tokens + self.k + 2
        tp = _pool_for(self.target, 1, cap, self.page_size)
        dp = _pool_for(self.draft, 1, cap, self.page_size)
        tp.allocate_sequence(0)
        dp.allocate_sequence(0)

        def pick(logits: torch.Tensor) -> Tuple[int, Optional[torch.Tensor]]:
            if temperature <= 0:
                return int(torch.argmax(logits)), None
            p = torch.softmax(logits / temperature, -1)
            return int(torch.multinomial(p.cpu(), 1, generator=g)), p

        lt = paged_logits(self.target, tp, [SeqChunk(0, 0, len(prompt))], prompt)[0]
        paged_logits(self.draft, dp, [SeqChunk(0, 0, len(prompt))], prompt)
        self.stats.target_forwards += 1
        last, _ = pick(lt)
        out = [last]
        ctx_len = len(prompt)  # tokens in both caches (``last`` is not cached yet)
        while len(out) < max_new_tokens and (eos_token_id is None or out[-1] != eos_token_id):
            k = min(self.k, max_new_tokens - len(out))
            # draft k tokens one at a time (its cache may lag by one token)
            dlen = dp.lengths[0]
            feed = (prompt + out)[dlen:ctx_len + 1]
            drafts, qs = [], []
            pos = dlen
            for _ in range(k):
                lg = paged_logits(self.draft, dp, [SeqChunk(0, pos, len(feed))], feed)[0]
                pos += len(feed)
                tok, q = pick(lg)
                drafts.append(tok)
                qs.append(q)
                feed = [tok]
            # verify: one chunk [last, d1..dk] on the target
            chunk = [last] + drafts
            lts = paged_logits(self.target, tp, [SeqChunk(0, ctx_len, len(chunk))], chunk,
                               all_positions=True)[0]
            self.stats.target_forwards += 1
            self.stats.drafted += k
            accepted = 0
            new_tok = None
            for i, d in enumerate(drafts):
                if temperature <= 0:
                    t = int(torch.argmax(lts[i]))
                    if t == d:
                        accepted += 1
                        continue
                    new_tok = t
                    break
                p = torch.softmax(lts[i] / temperature, -1)
                q = qs[i]
                if torch.rand((), generator=g) < min(1.0, float(p[d] / q[d].clamp_min(1e-20))):
                    accepted += 1
                    continue
                resid = (p - q.to(p.device)).clamp_min(0)
                resid = resid / resid.sum().clamp_min(1e-20)
                new_tok = int(torch.multinomial(resid.cpu(), 1, generator=g))
                break
            if new_tok is None:  # all accepted: bonus token from the last position
                new_tok, _ = pick(lts[k])
            self.stats.accepted += accepted
            out.extend(drafts[:accepted] + [new_tok])
            ctx_len += 1 + accepted
            tp.truncate_sequence(0, ctx_len)
            dp.truncate_sequence(0, min(dp.lengths[0], ctx_len))
            last = new_tok
            if eos_token_id is not None and eos_token_id in out:
                out = out[:out.index(eos_token_id) + 1]
                break
        return out[:max_new_tokens]


class SlidingWindowCache:
    """Contiguous per-layer KV cache that keeps only the last ``window`` tokens
    (``[L, B, Hkv, window, D]``); API of complexity/inference/kv_cache.py:331-429."""

    def __init__(self, num_layers: int, batch_size: int, num_heads: int, head_dim: int,
                 window: int, dtype=torch.float32, device="cpu"):
        shape = (num_layers, batch_size, num_heads, window, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.window = window
        self.filled = [0] * num_layers
        self.total = [0] * num_layers

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        n = k.shape[2]
        W = self.window
        if n >= W:
            self.k[layer] = k[:, :, -W:]
            self.v[layer] = v[:, :, -W:]
            self.filled[layer] = W
        else:
            f = self.filled[layer]
            if f + n > W:
                shift = f + n - W
                self.k[layer, :, :, :f - shift] = self.k[layer, :, :, shift:f].clone()
                self.v[layer, :, :, :f - shift] = self.v[layer, :, :, shift:f].clone()
                f -= shift
            self.k[layer, :, :, f:f + n] = k
            self.v[layer, :, :, f:f + n] = v
            self.filled[layer] = f + n
        self.total[layer] += n
        f = self.filled[layer]
        return self.k[layer, :, :, :f], self.v[layer, :, :, :f]

    def reset(self) -> None:
        self.filled = [0] * len(self.filled)
        self.total = [0] * len(self.total)

    @property
    def seq_len(self) -> int:
        return self.total[0]


# --------------------------------------------------- reference API names
@dataclass
class SpeculativeConfig:
    """complexity/inference/speculative.py:26-33."""
    num_speculative_tokens: int = 5
    acceptance_threshold: float = 0.0
    temperature: float = 1.0
    top_k: Optional[int] = None
    top_p: Optional[float] = None


class SelfSpeculativeDecoder:
    """Self-speculative decoding: the first ``exit_layer`` layers of the model
    (with its final norm and head) draft ``num_speculative_tokens`` tokens, the
    full model verifies them in one pass over the paged cache
    (complexity/inference/speculative.py:338-420)."""

    def __init__(self, model, exit_layer: int, config: Optional[SpeculativeConfig] = None,
                 page_size: int = 16):
        self.model, self.exit_layer = model, exit_layer
        self.config = config or SpeculativeConfig()
        self.decoder = SpeculativeDecoder(model, LayerSkipDraft(model, exit_layer),
                                          num_draft_tokens=self.config.num_speculative_tokens,
                                          page_size=page_size)

    def generate(self, input_ids, max_new_tokens: int = 100, eos_token_id: Optional[int] = None,
                 seed: Optional[int] = None):
        """``input_ids``: [1, T] tensor or a token list; returns the same kind."""
        as_tensor = torch.is_tensor(input_ids)
        prompt = input_ids.reshape(-1).tolist() if as_tensor else list(input_ids)
        temp = self.config.temperature if self.config.temperature != 1.0 or seed is not None \
            else 0.0
        out = self.decoder.generate(prompt, max_new_tokens=max_new_tokens, temperature=temp,
                                    eos_token_id=eos_token_id, seed=seed)
        seq = prompt + list(out)          # the decoder returns the new tokens only
        if as_tensor:
            return torch.tensor(seq, dtype=torch.long, device=input_ids.device)[None]
        return seq

    def get_statistics(self) -> dict:
        st = getattr(self.decoder, "stats", None)
        return dict(vars(st)) if st is not None else {}
