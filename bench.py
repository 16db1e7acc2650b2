"""Headline benchmark: TR-HASH 200M pretraining throughput (train tokens/s per box).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload decode ...   (7B paged-KV serving, bench_decode.py)
    python bench.py --workload ep1b|tp7b ... (1B expert-parallel / 7B tensor-parallel
                                              training, bench_train_large.py)

N > 1 is launched by torchrun (one process per GPU, NCCL).  Workload: the
released 200M TR-GQA/TR-Hash architecture, random init, synthetic Zipf(1.1)
token ids, seq 2048, micro-batch 16 per GPU, bf16 compute, AdamW with
grad-norm clipping, one optimizer step per micro-batch.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
``torch.cuda.synchronize()`` on both sides and timed with CUDA events on the
launching stream; the step time is the max over ranks.  Activations are GBs
per step, far larger than the 126 MB L2, so no explicit flush is needed.  A
second, end-to-end timed loop goes through the public ``Trainer.train_step``
API with the batch copied from pinned host memory every step and the loss
read back to the host every step.  SM clocks and throttle reasons are sampled
with nvidia-smi during the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
METRIC = "train tokens/s/box (max over ranks) TR-HASH 200M"
BASELINE_VALUE = None  # BASELINE.json publishes no number for this metric


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--seq", type=int, default=2048)
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-count", action="store_true", help="skip the kernel-launch count step")
    p.add_argument("--no-graph", action="store_true", help="run every step eagerly")
    p.add_argument("--zero3", action="store_true",
                   help="multi-GPU: ZeRO-3 (per-block parameter shards) instead of ZeRO-2")
    p.add_argument("--workload", choices=("train", "decode", "ep1b", "tp7b"), default="train",
                   help="train: the 200M pretraining headline; decode: 7B paged-KV serving; "
                        "ep1b: 1B expert-parallel training; tp7b: 7B tensor-parallel training")
    return p.parse_args()


def init_dist(n):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch N>1 with torchrun")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, (dist.get_rank() if world > 1 else 0), local


def zipf_batches(n_batches, B, S, V, seed, s=1.1):
    """Token ids with Zipf(s) frequencies over a seeded random rank->id map (pinned)."""
    g = torch.Generator().manual_seed(seed)
    ranks = torch.arange(1, V + 1, dtype=torch.float64)
    probs = ranks.pow(-s)
    probs /= probs.sum()
    order = torch.randperm(V, generator=g)
    out = []
    for _ in range(n_batches):
        r = torch.multinomial(probs, B * S, replacement=True, generator=g)
        out.append(order[r].view(B, S).pin_memory())
    return out


from complexity_framework_b200.profiling.timing import ClockSampler  # noqa: E402


def max_over_ranks(x, world):
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def timed(fn, steps, world):
    barrier(world)
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(steps):
        fn(i)
    e.record()
    barrier(world)
    return max_over_ranks(s.elapsed_time(e) / steps, world)


# ------------------------------------------------------------------ our arm
def build_ours(world, args):
    sys.path.insert(0, ROOT)
    from complexity_framework_b200 import ComplexityModel, tr_hash_200m_config
    from complexity_framework_b200.training import Trainer, TrainingConfig

    torch.manual_seed(0)
    model = ComplexityModel(tr_hash_200m_config())
    # steps after the second warm-up step replay a captured CUDA graph (forward +
    # backward + AdamW; on several GPUs also the fused NVLink reduce, whose barrier
    # epochs and hyper-parameters live on the device)
    cfg = TrainingConfig(learning_rate=3e-4, warmup_steps=0, lr_scheduler="constant",
                         precision="bf16", grad_clip=1.0, max_steps=10 ** 9,
                         distributed_mode=(("zero3" if args.zero3 else "fsdp") if world > 1
                                           else "none"),
                         skip_param_update_check=True,
                         cuda_graph=not args.no_graph, cuda_graph_warmup=2)
    trainer = Trainer(model, cfg)

    def step(ids, sync):
        return trainer.train_step(ids, sync=sync)

    if world == 1:
        mode = "single GPU, flat fp32-master fused AdamW" + (
            ", step replayed from a CUDA graph" if cfg.cuda_graph else "")
    elif args.zero3:
        mode = ("zero3 data parallel: per-block bf16 parameter shards gathered over NVLink one "
                "block ahead, gradient reduce-scatter overlapped with backward, sharded fp32 AdamW")
    else:
        mode = ("zero2 data parallel: fused NVLink gradient reduce + sharded fp32 AdamW "
                "(replicated bf16 params)" + (", step replayed from a CUDA graph"
                                               if cfg.cuda_graph else ""))
    return step, mode


def count_our_kernels(step_fn, ids):
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn(ids, False)
        torch.cuda.synchronize()
    ours = total = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            total += 1
            if "cfb::" in ev.name:
                ours += 1
    return ours, total


# ------------------------------------------------------------ reference arm
def build_reference(world, args):
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "complexity")):
        raise RuntimeError("reference not installed under baseline/_ref")
    sys.path.insert(0, ref_root)
    import complexity
    from complexity.core.losses import fused_linear_causal_lm_loss

    cfg = complexity.ModelConfig(
        hidden_size=896, num_hidden_layers=16, num_attention_heads=14, num_key_value_heads=2,
        intermediate_size=256, shared_intermediate_size=3072, vocab_size=32000,
        max_position_embeddings=2048, attention_type="gqa", mlp_type="tr_hash_engine",
        num_experts=4, top_k=2, top_k_primary_weight=0.5, routing_strategy="token_id_multi_hash",
        route_hash_count=2, shared_expert=True, shared_output_scale=1.0,
        routed_output_scale=2.0, use_qk_norm=True, tie_word_embeddings=True)
    torch.manual_seed(0)
    model = complexity.ComplexityModel(cfg).cuda()
    if world > 1:
        from complexity.parallel import wrap_model_fsdp

        model = wrap_model_fsdp(model)
        mode = "fsdp2 full_shard (reference wrap_model_fsdp, bf16 params)"
    else:
        mode = "single device (fp32 params + bf16 autocast, reference Trainer default)"
    decay = [p for n, p in model.named_parameters() if "norm" not in n and "bias" not in n]
    nodecay = [p for n, p in model.named_parameters() if "norm" in n or "bias" in n]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1},
                             {"params": nodecay, "weight_decay": 0.0}], lr=3e-4,
                            betas=(0.9, 0.95), foreach=False)

    def step(ids, sync):
        ids = ids.to("cuda", non_blocking=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = model(ids, return_logits=False)
            hidden = out["last_hidden_state"][:, :-1, :].contiguous()
            loss, _ = fused_linear_causal_lm_loss(hidden, model.embed_tokens.weight,
                                                  ids[:, 1:].contiguous(), sync_metrics=False)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return float(loss.detach()) if sync else loss.detach()

    return step, mode


def main():
    args = parse()
    world, rank, local = init_dist(args.gpus)
    if args.workload == "decode":
        sys.path.insert(0, ROOT)
        import bench_decode

        return bench_decode.main(args, world, rank, local, sys.modules[__name__])
    if args.workload in ("ep1b", "tp7b"):
        sys.path.insert(0, ROOT)
        import bench_train_large

        bench_train_large.main(args, world, rank, local, sys.modules[__name__])
        if world > 1:
            dist.destroy_process_group()
        return
    B, S, V = args.batch, args.seq, 32000
    try:
        build = build_ours if args.impl == "ours" else build_reference
        step, mode = build(world, args)
    except Exception as exc:
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: "
                                  f"{str(exc).splitlines()[0] if str(exc) else ''}"}))
            return
        raise
    host = zipf_batches(4, B, S, V, seed=1234 + rank)
    dev = [h.to("cuda") for h in host]
    for i in range(args.warmup):
        step(dev[i % 4], False)
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    if local == 0:
        clocks.start()
    ms = timed(lambda i: step(dev[i % 4], False), args.steps, world)
    clk = clocks.stop() if local == 0 else None

    e2e = None
    if not args.no_e2e:
        k2 = args.e2e_steps or args.steps
        t0 = time.perf_counter()
        ms_e2e = timed(lambda i: step(host[i % 4], True), k2, world)
        wall = (time.perf_counter() - t0) / k2 * 1000
        e2e = {"value": B * S * world / (ms_e2e / 1000.0), "unit": "tokens/s",
               "ms_per_step": ms_e2e, "wall_ms_per_step": wall,
               "h2d_bytes_per_step": host[0].numel() * host[0].element_size(),
               "d2h_bytes_per_step": 4,
               "api": ("complexity_framework_b200.training.Trainer.train_step" if
                       args.impl == "ours" else "reference model + fused_linear_causal_lm_loss")}

    launches = None
    if args.impl == "ours" and not args.no_count:
        ours, total = count_our_kernels(step, dev[0])
        launches = ours * args.steps
        launches_total = total * args.steps
    value = B * S * world / (ms / 1000.0)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None,
            "dtype": "bf16", "data": "synthetic Zipf(1.1) token ids, random-init weights",
            "config": {"model": "TR-HASH 200M (16L, H896, GQA 14/2, 4 experts W64 top-2 "
                                "multi-hash, shared 3072, V32000)",
                       "global_batch": B * world, "micro_batch_per_gpu": B, "seq_len": S,
                       "parallelism": f"dp{world}", "mode": mode,
                       "l2": "inputs/activations larger than L2 (no flush needed)"},
            "clocks": clk, "e2e": e2e,
        }
        if args.impl == "ours":
            if launches is not None:
                line["gpu_launches"] = launches
                line["gpu_launches_all"] = launches_total
        else:
            line["impl"] = "reference"
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
