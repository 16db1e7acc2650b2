"""Paged-KV inference engine with continuous batching.

Every engine step runs ONE forward over a ragged batch: the pending prompt
chunks (chunked prefill, bounded by ``max_tokens_per_step``) and one decode
token for every running request, concatenated into ``[1, N, H]``.  Attention
reads each sequence's pages in place (``inference.paged``); the MLP, norms and
projections run the same fused sm_100a kernels as training.  Requests join
and leave between steps; their pages return to the pool when they finish.

API names follow complexity/inference/engine.py:25-709 (``DecodingStrategy``,
``GenerationConfig``, ``InferenceConfig``, ``InferenceEngine.generate``,
``generate_stream``, ``generate_batch``, ``add_request``/``step_serving``).
Unlike the reference (whose paged engine cannot run) the cache
is wired into the model.
"""
from __future__ import annotations

import itertools
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, Iterator, List, Optional, Sequence, Union

import torch

from .paged import PagedBatch, PagePool, SeqChunk


class DecodingStrategy(Enum):
    GREEDY = "greedy"
    SAMPLING = "sampling"
    BEAM_SEARCH = "beam_search"
    TOP_K = "top_k"
    TOP_P = "top_p"
    CONTRASTIVE = "contrastive"


@dataclass
class GenerationConfig:
    max_new_tokens: int = 100
    min_new_tokens: int = 0
    strategy: DecodingStrategy = DecodingStrategy.GREEDY
    do_sample: bool = False
    temperature: float = 1.0
    top_k: Optional[int] = 0
    top_p: Optional[float] = 1.0
    num_beams: int = 1
    repetition_penalty: float = 1.0
    no_repeat_ngram_size: int = 0
    eos_token_id: Optional[int] = None
    pad_token_id: Optional[int] = None
    stop_sequences: Optional[List[List[int]]] = None
    seed: Optional[int] = None

    @property
    def sampling(self) -> bool:
        return self.do_sample or self.strategy in (DecodingStrategy.SAMPLING,
                                                   DecodingStrategy.TOP_K, DecodingStrategy.TOP_P)


@dataclass
class InferenceConfig:
    use_kv_cache: bool = True
    cache_type: str = "paged"
    max_cache_length: int = 4096
    page_size: int = 16
    num_pages: Optional[int] = None          # default: max_batch_size * max_cache_length / page
    max_batch_size: int = 64
    max_tokens_per_step: int = 8192
    prefill_chunk_size: int = 2048
    dtype: Optional[torch.dtype] = None
    device: Optional[torch.device] = None
    # decode-only steps of greedy requests replay a captured CUDA graph per
    # padded batch size (CUDA only)
    cuda_graph_decode: bool = True
    decode_graph_buckets: Sequence[int] = (1, 2, 4, 8, 16, 32, 64, 128, 256)


@dataclass
class _Req:
    rid: int
    prompt: List[int]
    gen: GenerationConfig
    output: List[int] = field(default_factory=list)
    prefilled: int = 0
    done: bool = False
    arrival: float = 0.0
    first_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    generator: Optional[torch.Generator] = None


def plain_greedy(gen: GenerationConfig) -> bool:
    """Greedy decoding with no history-dependent logit processing: the next
    token is the argmax, so a whole batch is selected on the device at once."""
    return (not gen.sampling or gen.temperature <= 0) and gen.repetition_penalty == 1.0 \
        and gen.no_repeat_ngram_size == 0


def sample_next(logits: torch.Tensor, gen: GenerationConfig, history: Sequence[int],
                generator: Optional[torch.Generator] = None) -> int:
    """One token from a [V] logit row (greedy, temperature, top-k, top-p, penalties)."""
    logits = logits.float()
    if gen.repetition_penalty != 1.0 and history:
        idx = torch.tensor(sorted(set(history)), device=logits.device)
        vals = logits[idx]
        logits[idx] = torch.where(vals > 0, vals / gen.repetition_penalty,
                                  vals * gen.repetition_penalty)
    n = gen.no_repeat_ngram_size
    if n > 0 and len(history) >= n - 1:
        prefix = tuple(history[len(history) - n + 1:]) if n > 1 else tuple()
        banned = {history[i + n - 1] for i in range(len(history) - n + 1)
                  if tuple(history[i:i + n - 1]) == prefix}
        if banned:
            logits[torch.tensor(sorted(banned), device=logits.device)] = float("-inf")
    if not gen.sampling or gen.temperature <= 0:
        return int(torch.argmax(logits))
    logits = logits / gen.temperature
    if gen.top_k:
        kth = torch.topk(logits, min(gen.top_k, logits.numel())).values[-1]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if gen.top_p is not None and gen.top_p < 1.0:
        sl, si = torch.sort(logits, descending=True)
        cp = torch.softmax(sl, -1).cumsum(-1)
        drop = cp - torch.softmax(sl, -1) > gen.top_p
        sl = sl.masked_fill(drop, float("-inf"))
        logits = torch.full_like(logits, float("-inf")).scatter(0, si, sl)
    probs = torch.softmax(logits, -1)
    return int(torch.multinomial(probs.cpu(), 1, generator=generator))


@torch.no_grad()
def forward_paged(model, ids: torch.Tensor, batch: PagedBatch) -> torch.Tensor:
    """Final-norm hidden states [N, H] of the N new tokens (``ids`` is [N])."""
    tok = ids.view(1, -1)
    x = model.embed(tok)
    pe = getattr(model, "embed_positions", None)
    if pe is not None:
        x = x + pe.weight[batch.positions].to(x.dtype)[None]
    for layer in model.layers:
        x = layer.forward_paged(x, batch, tok)
    return model.norm(x)[0]


class InferenceEngine:
    def __init__(self, model, config: Optional[InferenceConfig] = None):
        self.model = model.eval()
        self.config = config or InferenceConfig()
        p = next(model.parameters())
        self.device = self.config.device or p.device
        self.dtype = self.config.dtype or p.dtype
        mc = model.config
        pages = self.config.num_pages or (
            self.config.max_batch_size * self.config.max_cache_length // self.config.page_size)
        # KV heads held by this rank (fewer than the config's under tensor parallelism)
        kv_heads = getattr(getattr(model.layers[0], "self_attn", None), "num_kv_heads",
                           mc.num_key_value_heads)
        self.pool = PagePool(mc.num_hidden_layers, kv_heads, mc.head_dim, pages,
                             self.config.page_size, dtype=self.dtype, device=self.device)
        self._ids = itertools.count()
        self._graphs: Dict[int, tuple] = {}
        self.requests: Dict[int, _Req] = {}
        self.waiting: List[int] = []
        self.running: List[int] = []
        self.stats = {"steps": 0, "tokens_prefilled": 0, "tokens_decoded": 0}

    # ------------------------------------------------------------ requests
    def add_request(self, prompt: Union[Sequence[int], torch.Tensor],
                    generation_config: Optional[GenerationConfig] = None) -> int:
        ids = prompt.tolist() if isinstance(prompt, torch.Tensor) else list(prompt)
        if not ids:
            raise ValueError("empty prompt")
        gen = generation_config or GenerationConfig()
        rid = next(self._ids)
        g = None
        if gen.seed is not None:
            g = torch.Generator().manual_seed(int(gen.seed) + rid)
        self.requests[rid] = _Req(rid, ids, gen, arrival=time.perf_counter(), generator=g)
        self.waiting.append(rid)
        return rid

    def has_pending(self) -> bool:
        return bool(self.waiting or self.running)

    def _finish(self, r: _Req) -> None:
        r.done = True
        r.finish_time = time.perf_counter()
        self.pool.free_sequence(r.rid)

    def _stop(self, r: _Req, tok: int) -> bool:
        g = r.gen
        if len(r.output) >= g.max_new_tokens:
            return True
        if len(r.output) < g.min_new_tokens:
            return False
        if g.eos_token_id is not None and tok == g.eos_token_id:
            return True
        for seq in g.stop_sequences or []:
            if seq and r.output[-len(seq):] == list(seq):
                return True
        return len(r.prompt) + len(r.output) >= self.config.max_cache_length

    # ---------------------------------------------------------------- step
    # --------------------------------------------------- graph-replayed decode
    def _graph_eligible(self) -> bool:
        return (self.config.cuda_graph_decode and self.device.type == "cuda" and bool(self.running)
                and not self.waiting and all(plain_greedy(self.requests[r].gen)
                                             for r in self.running)
                and len(self.running) <= max(self.config.decode_graph_buckets))

    def _decode_graph(self, size: int):
        """(static batch, graph, next-token buffer) for a padded decode batch."""
        from .paged import StaticDecodeBatch

        got = self._graphs.get(size)
        if got is not None:
            return got
        cfg = self.config
        max_pages = -(-cfg.max_cache_length // cfg.page_size)
        sb = StaticDecodeBatch(self.pool, size, max_pages, cfg.max_cache_length - 1)
        sb.fill([])

        def body():
            sb.expand()
            hidden = forward_paged(self.model, sb.ids, sb)
            return self.model.logits(hidden[None])[0].argmax(-1)

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # lazy initialisation outside the capture
            body()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = body()
        got = (sb, g, out)
        self._graphs[size] = got
        return got

    def warmup_decode_graphs(self, max_batch: Optional[int] = None) -> List[int]:
        """Capture the decode graph of every bucket up to ``max_batch`` (default:
        ``max_batch_size``) now, so no capture lands inside serving."""
        if not (self.config.cuda_graph_decode and self.device.type == "cuda"):
            return []
        limit = max_batch or self.config.max_batch_size
        sizes = [b for b in self.config.decode_graph_buckets if b <= limit]
        bigger = [b for b in self.config.decode_graph_buckets if b > limit]
        if bigger and (not sizes or sizes[-1] < limit):
            sizes.append(bigger[0])
        with torch.no_grad():
            for b in sizes:
                self._decode_graph(b)
        return sizes

    def _graph_decode_step(self) -> List[int]:
        rids = list(self.running)
        size = min(b for b in self.config.decode_graph_buckets if b >= len(rids))
        sb, graph, out = self._decode_graph(size)
        entries = []
        for rid in rids:
            r = self.requests[rid]
            entries.append((rid, r.output[-1], len(r.prompt) + len(r.output) - 1))
        sb.fill(entries)
        graph.replay()
        toks = out[:len(rids)].tolist()   # the step's only device-to-host read
        sb.commit()
        finished = []
        for rid, tok in zip(rids, toks):
            r = self.requests[rid]
            r.output.append(int(tok))
            if self._stop(r, int(tok)):
                self._finish(r)
                self.running.remove(rid)
                finished.append(rid)
        self.stats["steps"] += 1
        self.stats["tokens_decoded"] += len(rids)
        self.stats["graph_steps"] = self.stats.get("graph_steps", 0) + 1
        return finished

    @torch.no_grad()
    def step(self) -> List[int]:
        """Run one batched forward; returns ids of requests that finished."""
        if self._graph_eligible():
            return self._graph_decode_step()
        budget = self.config.max_tokens_per_step
        chunks: List[SeqChunk] = []
        toks: List[int] = []
        owners: List[_Req] = []
        for rid in list(self.running):
            r = self.requests[rid]
            pos = len(r.prompt) + len(r.output) - 1
            chunks.append(SeqChunk(rid, pos, 1))
            toks.append(r.output[-1])
            owners.append(r)
            budget -= 1
        while self.waiting and budget > 0 and len(self.running) < self.config.max_batch_size:
            r = self.requests[self.waiting[0]]
            if r.prefilled == 0 and r.rid not in self.pool.pages:
                if not self.pool.can_reserve(None, min(len(r.prompt), self.config.max_cache_length)):
                    break
                self.pool.allocate_sequence(r.rid)
            n = min(len(r.prompt) - r.prefilled, budget, self.config.prefill_chunk_size)
            chunks.append(SeqChunk(r.rid, r.prefilled, n))
            toks.extend(r.prompt[r.prefilled:r.prefilled + n])
            owners.append(r)
            r.prefilled += n
            budget -= n
            if r.prefilled == len(r.prompt):
                self.waiting.pop(0)
                self.running.append(r.rid)
            else:
                break
        if not chunks:
            return []
        batch = PagedBatch(self.pool, chunks)
        ids = torch.tensor(toks, dtype=torch.long, device=self.device)
        hidden = forward_paged(self.model, ids, batch)
        batch.commit()
        last = torch.tensor([c - 1 for c in batch._cu_host[1:]], device=self.device)
        logits = self.model.logits(hidden[last][None])[0]
        finished = []
        # greedy rows: one argmax over the batch and a single device-to-host read
        greedy = None
        if all(plain_greedy(r.gen) for r in owners):
            greedy = logits.argmax(-1).tolist()
        now = time.perf_counter()
        for i, (c, r) in enumerate(zip(chunks, owners)):
            if c.start + c.length < len(r.prompt):
                continue  # mid-prompt chunk: no token yet
            tok = (greedy[i] if greedy is not None
                   else sample_next(logits[i], r.gen, r.prompt + r.output, r.generator))
            r.output.append(tok)
            if r.first_token_time is None:
                r.first_token_time = now
            if self._stop(r, tok):
                self._finish(r)
                if r.rid in self.running:
                    self.running.remove(r.rid)
                finished.append(r.rid)
        self.stats["steps"] += 1
        self.stats["tokens_decoded"] += sum(1 for c in chunks if c.length == 1)
        self.stats["tokens_prefilled"] += sum(c.length for c in chunks if c.length > 1)
        return finished

    # ------------------------------------------------------------- front ends
    def generate_tokens(self, prompts: Sequence[Sequence[int]],
                        generation_config: Optional[GenerationConfig] = None) -> List[List[int]]:
        rids = [self.add_request(p, generation_config) for p in prompts]
        while any(not self.requests[r].done for r in rids):
            self.step()
        outs = [self.requests[r].output for r in rids]
        for r in rids:
            self.requests.pop(r, None)
        return outs

    def generate(self, input_ids, generation_config: Optional[GenerationConfig] = None,
                 attention_mask: Optional[torch.Tensor] = None):
        """Prompt(s) -> {"sequences": prompt+generated per row, "new_tokens": generated}.

        ``input_ids`` may be a [B, S] tensor (``attention_mask`` zeros mark left
        or right padding to strip) or a list of token lists.
        """
        if isinstance(input_ids, torch.Tensor):
            rows = []
            for b in range(input_ids.shape[0]):
                row = input_ids[b]
                if attention_mask is not None:
                    row = row[attention_mask[b].bool()]
                rows.append(row.tolist())
        else:
            rows = [list(r) for r in input_ids]
        new = self.generate_tokens(rows, generation_config)
        return {"sequences": [r + n for r, n in zip(rows, new)], "new_tokens": new}

    def generate_stream(self, prompt: Sequence[int],
                        generation_config: Optional[GenerationConfig] = None) -> Iterator[int]:
        rid = self.add_request(prompt, generation_config)
        seen = 0
        while not self.requests[rid].done:
            self.step()
            out = self.requests[rid].output
            while seen < len(out):
                yield out[seen]
                seen += 1
        out = self.requests.pop(rid).output
        while seen < len(out):
            yield out[seen]
            seen += 1

    def generate_batch(self, prompts: Sequence[Sequence[int]],
                       generation_config: Optional[GenerationConfig] = None) -> List[List[int]]:
        return self.generate_tokens(prompts, generation_config)

    # serving-style API
    def start_serving(self) -> None:
        self.stats = {"steps": 0, "tokens_prefilled": 0, "tokens_decoded": 0}

    def step_serving(self) -> List[Dict]:
        done = self.step()
        out = []
        for rid in done:
            r = self.requests[rid]
            out.append({"request_id": rid, "output_ids": list(r.output),
                        "ttft_s": (r.first_token_time or r.finish_time) - r.arrival,
                        "latency_s": r.finish_time - r.arrival})
        return out

    def get_serving_stats(self) -> Dict:
        return dict(self.stats, running=len(self.running), waiting=len(self.waiting),
                    **self.pool.memory_usage())
