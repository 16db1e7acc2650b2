"""Serving benchmark: TR-GQA 7B greedy decode through the paged-KV engine.

    python bench.py --workload decode [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: 64 concurrent requests, prompt lengths uniform in [128, 2048]
with uniform random token ids (seeded), 256 greedy tokens each, KV page size
16, bf16 weights with random init.  Architecture: 32 layers, hidden 4096, GQA
32/8 (head_dim 128), vocab 32000, shared SwiGLU 11008, 8 routed experts of
width 512, top-2 modulo_cyclic.

A "step" is one complete serving run of the 64 requests (prefill and decode);
a warm-up step runs the same prompts with 8 new tokens.  Reported:

* ``value``: decode tokens/s over the decode phase (from the first step with
  no prompt left to prefill to the end), timed with CUDA events, max over
  ranks; with N GPUs the model is tensor parallel over all N (every rank runs
  the same engine schedule on its shard), so the work is fixed ("strong");
* ``ttft_p50_ms``: median time from submission to a request's first token;
* ``e2e``: the same decode rate on the host clock, through the public engine
  API, with prompts handed over as host lists and every step's tokens read
  back to the host.

The reference arm drives the reference model's own KV-cache API
(``model(ids, past_key_values=..., use_cache=True)``): all prompts left-padded
into one batch, one prefill, then one batched forward per token.  Its
``InferenceEngine.generate`` does not pass the cache back to the model and its
``ContinuousBatcher`` recomputes every sequence each step, so neither is a
KV-cached decode; the padded batch is the fastest cached path it offers.
"""
from __future__ import annotations

import json
import os
import statistics
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode tokens/s TR-GQA 7B paged-KV engine (tensor parallel over the GPUs)"
N_REQ, NEW_TOKENS, PROMPT_MIN, PROMPT_MAX, PAGE = 64, 256, 128, 2048, 16
ARCH = dict(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
            num_key_value_heads=8, intermediate_size=4096, shared_intermediate_size=11008,
            vocab_size=32000, num_experts=8, top_k=2, routing_strategy="modulo_cyclic",
            attention_type="gqa", mlp_type="tr_hash_engine", shared_expert=True,
            max_position_embeddings=4096, tie_word_embeddings=False)


def prompts(seed: int):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(PROMPT_MIN, PROMPT_MAX + 1, (N_REQ,), generator=g).tolist()
    return [torch.randint(0, ARCH["vocab_size"], (n,), generator=g).tolist() for n in lens]


# ------------------------------------------------------------------ our arm
class OursDecode:
    def __init__(self, world: int = 1):
        sys.path.insert(0, ROOT)
        from complexity_framework_b200 import ComplexityModel, ModelConfig
        from complexity_framework_b200.inference.engine import InferenceConfig, InferenceEngine

        torch.manual_seed(0)
        with torch.device("cuda"):
            model = ComplexityModel(ModelConfig(**ARCH))
        # route tables are built on the host; move them with everything else
        self.model = model.to("cuda").to(torch.bfloat16).eval()
        self.tp = world
        if world > 1:
            import torch.distributed as dist

            from complexity_framework_b200.parallel.tp_inference import enable_tp_decode

            enable_tp_decode(self.model, dist.group.WORLD)
            torch.cuda.empty_cache()
        self.cfg = InferenceConfig(max_cache_length=PROMPT_MAX + NEW_TOKENS, page_size=PAGE,
                                   max_batch_size=N_REQ, max_tokens_per_step=8192,
                                   prefill_chunk_size=2048)
        self.engine = InferenceEngine(self.model, self.cfg)
        self.graph_sizes = self.engine.warmup_decode_graphs(N_REQ)
        self.mode = ("paged-KV engine, chunked prefill, decode steps replayed from CUDA graphs "
                     f"(buckets {self.graph_sizes})")
        if world > 1:
            comm = self.model.tp_decode
            self.mode += (f"; tensor parallel x{world}: fused peer-memory all-reduce + residual "
                          f"per attention and FFN ({'NVLS multimem' if comm.uses_multicast else 'unicast'})")

    def run(self, ps, new_tokens):
        from complexity_framework_b200.inference.engine import GenerationConfig

        eng = self.engine
        gen = GenerationConfig(max_new_tokens=new_tokens, do_sample=False)
        torch.cuda.synchronize()
        ev0, ev_dec, ev1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        t0 = time.perf_counter()
        ev0.record()
        rids = [eng.add_request(p, gen) for p in ps]
        dec_tokens0 = None
        t_dec = None
        steps = 0
        while eng.has_pending():
            if dec_tokens0 is None and not eng.waiting:
                ev_dec.record()
                t_dec = time.perf_counter()
                dec_tokens0 = sum(len(eng.requests[r].output) for r in rids)
            eng.step()
            steps += 1
        ev1.record()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        total = sum(len(eng.requests[r].output) for r in rids)
        ttft = [(eng.requests[r].first_token_time - eng.requests[r].arrival) * 1000 for r in rids]
        for r in rids:
            eng.requests.pop(r, None)
        return {"decode_tokens": total - dec_tokens0, "total_tokens": total,
                "decode_ms": ev_dec.elapsed_time(ev1), "total_ms": ev0.elapsed_time(ev1),
                "decode_wall_ms": (t1 - t_dec) * 1000, "total_wall_ms": (t1 - t0) * 1000,
                "ttft_p50_ms": statistics.median(ttft), "steps": steps}

    def count_launches(self):
        """(our kernels, all kernels) in one replayed decode step of the full batch."""
        from torch.profiler import ProfilerActivity, profile

        sb, graph, _ = self.engine._decode_graph(self.graph_sizes[-1])
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            graph.replay()
            torch.cuda.synchronize()
        ours = total = 0
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                total += 1
                ours += "cfb::" in ev.name
        return ours, total

    def io_bytes(self):
        sb = self.engine._decode_graph(self.graph_sizes[-1])[0]
        return sb.host.numel() * sb.host.element_size(), N_REQ * 8


# ------------------------------------------------------------ reference arm
class ReferenceDecode:
    def __init__(self, world: int = 1):
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "complexity")):
            raise RuntimeError("reference not installed under baseline/_ref")
        sys.path.insert(0, ref_root)
        import complexity

        torch.manual_seed(0)
        with torch.device("cuda"):
            model = complexity.ComplexityModel(complexity.ModelConfig(**ARCH))
        # route tables are built on the host; move them with everything else
        self.model = model.to("cuda").to(torch.bfloat16).eval()
        self.mode = ("reference model KV-cache API: left-padded batch, one prefill, "
                     "one batched forward per token")
        if world > 1:
            from complexity.parallel.tensor_parallel import (init_tensor_parallel_group,
                                                             make_parallel)

            init_tensor_parallel_group(world)
            make_parallel(self.model, world)
            # its parallel layers are created on the host: move them over
            self.model = self.model.to("cuda").to(torch.bfloat16)
            torch.cuda.empty_cache()
            self.mode += f"; reference make_parallel tensor parallel x{world} (attention sharded)"

    @torch.no_grad()
    def run(self, ps, new_tokens):
        L = max(len(p) for p in ps)
        pad = torch.zeros(len(ps), L, dtype=torch.long).pin_memory()
        for i, p in enumerate(ps):
            pad[i, L - len(p):] = torch.tensor(p)
        torch.cuda.synchronize()
        ev0, ev_dec, ev1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        t0 = time.perf_counter()
        ev0.record()
        ids = pad.to("cuda", non_blocking=True)
        out = self.model(ids, use_cache=True)
        pkv = out["past_key_values"]
        tok = out["logits"][:, -1].argmax(-1)
        toks = [tok.tolist()]
        ttft = (time.perf_counter() - t0) * 1000
        del out
        ev_dec.record()
        t_dec = time.perf_counter()
        for _ in range(new_tokens - 1):
            out = self.model(tok[:, None], past_key_values=pkv, use_cache=True)
            pkv = out["past_key_values"]
            tok = out["logits"][:, -1].argmax(-1)
            toks.append(tok.tolist())
        ev1.record()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        n = len(ps)
        return {"decode_tokens": n * (new_tokens - 1), "total_tokens": n * new_tokens,
                "decode_ms": ev_dec.elapsed_time(ev1), "total_ms": ev0.elapsed_time(ev1),
                "decode_wall_ms": (t1 - t_dec) * 1000, "total_wall_ms": (t1 - t0) * 1000,
                "ttft_p50_ms": ttft, "steps": new_tokens}


def main(args, world, rank, local, helpers):
    """Run the decode workload; ``helpers`` is the bench module (clock sampler,
    max-over-ranks reduction)."""
    import torch.distributed as dist

    try:
        arm = OursDecode(world) if args.impl == "ours" else ReferenceDecode(world)
    except Exception as exc:
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: "
                                  f"{str(exc).splitlines()[0] if str(exc) else ''}"}))
            return
        raise
    ps = prompts(4321)  # tensor parallel: every rank serves the same requests
    for _ in range(args.warmup):
        arm.run(ps, 8)
    helpers.barrier(world)
    clocks = helpers.ClockSampler(local)
    if local == 0:
        clocks.start()
    runs = []
    for _ in range(args.steps):
        helpers.barrier(world)
        runs.append(arm.run(ps, NEW_TOKENS))
    helpers.barrier(world)
    clk = clocks.stop() if local == 0 else None

    dec_ms = helpers.max_over_ranks(sum(r["decode_ms"] for r in runs), world)
    dec_wall = helpers.max_over_ranks(sum(r["decode_wall_ms"] for r in runs), world)
    tot_wall = helpers.max_over_ranks(sum(r["total_wall_ms"] for r in runs), world)
    ttft = helpers.max_over_ranks(statistics.median(r["ttft_p50_ms"] for r in runs), world)
    dec_tokens = sum(r["decode_tokens"] for r in runs)
    tot_tokens = sum(r["total_tokens"] for r in runs)
    value = dec_tokens / (dec_ms / 1000.0)
    launches = None
    if args.impl == "ours" and not args.no_count:
        ours, total = arm.count_launches()
        launches = (ours, total, sum(r["steps"] for r in runs))
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dec_ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: uniform random prompt ids, lengths U[128,2048], random-init weights",
            "config": {"model": "TR-GQA 7B (32L, H4096, GQA 32/8, shared 11008, 8 experts W512 "
                                "top-2 modulo_cyclic, V32000)",
                       "requests": N_REQ, "new_tokens": NEW_TOKENS,
                       "prompt_len": [PROMPT_MIN, PROMPT_MAX], "page_size": PAGE,
                       "parallelism": f"tp{world}", "mode": arm.mode,
                       "l2": "15 GB of weights read per decode step (no flush needed)"},
            "ttft_p50_ms": ttft,
            "output_tokens_per_s_incl_prefill": tot_tokens / (tot_wall / 1000.0),
            "clocks": clk,
        }
        e2e = {"value": dec_tokens / (dec_wall / 1000.0), "unit": "tokens/s",
               "api": ("complexity_framework_b200.inference.InferenceEngine.add_request/step"
                       if args.impl == "ours" else "reference ComplexityModel forward with "
                       "past_key_values")}
        if args.impl == "ours":
            h2d, d2h = arm.io_bytes()
            e2e.update(h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h)
            if launches is not None:
                line["gpu_launches"] = launches[0] * launches[2]
                line["gpu_launches_per_decode_step"] = launches[0]
                line["gpu_kernels_per_decode_step"] = launches[1]
        else:
            e2e.update(h2d_bytes_per_step=8 * N_REQ, d2h_bytes_per_step=8 * N_REQ)
            line["impl"] = "reference"
        line["e2e"] = e2e
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
