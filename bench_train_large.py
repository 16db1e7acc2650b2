"""Training benchmarks of the two large BASELINE configs.

    python bench.py --workload ep1b [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload tp7b  ...

``ep1b``: TR-GQA 1B, expert parallel over the N GPUs (16 routed experts of
width 256, so 2 per GPU at N=8), 24 layers, hidden 2048, GQA 16/4 (head_dim
128), shared SwiGLU 5632, top-2 token_id_balanced_hash, seq 2048,
micro-batch 8 per GPU, Zipf(1.1) token ids.  Ours: the routed experts sharded
over the ranks with NVLink pull dispatch/combine fused around the grouped
tcgen05 expert GEMMs (``parallel/ep_fused.py``), token ids gathered once per
forward; the replicated parameters are data parallel (NCCL reduce-scatter,
sharded fp32 AdamW, all-gather).  Per-GPU work is fixed ("weak").  The
reference has no expert parallelism: its arm runs the same model under its
own ``ClusterModel`` data parallel in DDP mode (N > 1) with every expert on
every rank (its FSDP mode fails in its Triton grouped GEMM on this config:
fp32 activations against bf16 expert weights).

``tp7b``: TR-MHA 7B, 32 layers, hidden 4096, 32 MHA heads (head_dim 128),
shared SwiGLU 11008, 8 routed experts of width 512, top-2 modulo_cyclic, seq
4096, micro-batch 2, uniform random ids, tensor parallel over all N GPUs
(the FSDP dimension is 1 on one box of 8).  Ours: sequence-parallel TP with
the all-gather inside the first GEMM of attention and of the FFN and the
reduce-scatter as local partials plus an NVLink finish kernel
(``parallel/tp_fused.py``); attention heads, the shared SwiGLU and every
expert's width are sharded.  The whole job trains one micro-batch per step
("strong").  The reference arm is its ``ClusterModel(tp_size=N)``: attention
sharded, the FFN replicated, bf16 parameters (fp32 would not fit its
replicated FFN and optimizer state).  7B does not fit one GPU with fp32
master weights and moments, so ``tp7b`` needs N >= 2.

Timing as in ``bench.py``: W warm-up steps, K steps bracketed by barriers and
``torch.cuda.synchronize()``, CUDA events, max over ranks, clocks sampled
during the timed loop; an end-to-end loop through ``Trainer.train_step``
copies each step's batch from pinned host memory and reads the loss back.
Multi-GPU steps of both workloads run eagerly (no CUDA graph).
"""
from __future__ import annotations

import json
import os
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))

EP1B = dict(hidden_size=2048, num_hidden_layers=24, num_attention_heads=16,
            num_key_value_heads=4, intermediate_size=16 * 256, shared_intermediate_size=5632,
            vocab_size=32000, num_experts=16, top_k=2, routing_strategy="token_id_balanced_hash",
            attention_type="gqa", mlp_type="tr_hash_engine", shared_expert=True,
            max_position_embeddings=2048)
TP7B = dict(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
            num_key_value_heads=32, intermediate_size=8 * 512, shared_intermediate_size=11008,
            vocab_size=32000, num_experts=8, top_k=2, routing_strategy="modulo_cyclic",
            attention_type="mha", mlp_type="tr_hash_engine", shared_expert=True,
            max_position_embeddings=4096)

SPEC = {
    "ep1b": dict(arch=EP1B, batch=8, seq=2048, zipf=True, scaling="weak",
                 metric="train tokens/s/box (max over ranks) TR-GQA 1B expert parallel",
                 model="TR-GQA 1B (24L, H2048, GQA 16/4, shared 5632, 16 experts W256 top-2 "
                       "balanced hash, V32000)"),
    "tp7b": dict(arch=TP7B, batch=2, seq=4096, zipf=False, scaling="strong",
                 metric="train tokens/s/box (max over ranks) TR-MHA 7B tensor parallel",
                 model="TR-MHA 7B (32L, H4096, MHA 32, shared 11008, 8 experts W512 top-2 "
                       "modulo_cyclic, V32000)"),
}


def _uniform(n, B, S, V, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, V, (B, S), generator=g).pin_memory() for _ in range(n)]


def build_ours(workload, world):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.training import Trainer, TrainingConfig

    spec = SPEC[workload]
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = ComplexityModel(ModelConfig(**spec["arch"]))
    model = model.to("cuda").to(torch.bfloat16)
    graph = False
    if workload == "ep1b":
        if world > 1:
            from complexity_framework_b200.parallel.ep_fused import make_fused_expert_parallel

            make_fused_expert_parallel(model, dist.group.WORLD)
            mode = (f"expert parallel x{world} ({16 // world} experts/GPU): NVLink pull "
                    "dispatch/combine around grouped tcgen05 expert GEMMs; replicated "
                    "parameters data parallel (NCCL reduce-scatter, sharded fp32 AdamW)")
            dmode = "fsdp"
        else:
            mode = ("single GPU, all 16 experts local on the grouped tcgen05 expert GEMMs, "
                    "step replayed from a CUDA graph")
            dmode, graph = "none", True
    else:
        if world < 2:
            raise RuntimeError("TR-MHA 7B training needs tensor parallelism over >= 2 GPUs "
                               "(fp32 master weights and moments exceed one GPU)")
        from complexity_framework_b200.parallel.tp_fused import enable_fused_sequence_parallel

        enable_fused_sequence_parallel(model, dist.group.WORLD)
        torch.cuda.empty_cache()
        mode = (f"tensor parallel x{world}, sequence parallel: all-gather fused into the "
                "QKV and gate|up GEMMs, GEMM partials reduce-scattered by an NVLink finish "
                "kernel; heads, shared SwiGLU and expert widths sharded")
        dmode = "none"
    cfg = TrainingConfig(learning_rate=3e-4, warmup_steps=0, lr_scheduler="constant",
                         precision="bf16", grad_clip=1.0, max_steps=10 ** 9,
                         distributed_mode=dmode, skip_param_update_check=True,
                         cuda_graph=graph, cuda_graph_warmup=2)
    trainer = Trainer(model, cfg)

    def step(ids, sync):
        return trainer.train_step(ids, sync=sync)

    return step, mode


def build_reference(workload, world):
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "complexity")):
        raise RuntimeError("reference not installed under baseline/_ref")
    sys.path.insert(0, ref_root)
    import complexity
    from complexity.core.losses import fused_linear_causal_lm_loss

    spec = SPEC[workload]
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = complexity.ComplexityModel(complexity.ModelConfig(**spec["arch"]))
    model = model.to("cuda")
    autocast = True
    if workload == "ep1b":
        if world > 1:
            # its FSDP arm (bf16 parameters) fails in the CGGR Triton grouped GEMM
            # on this config (fp32 activations against bf16 expert weights), so
            # the reference's DDP mode runs: fp32 parameters under bf16 autocast
            from complexity.parallel.cluster import ClusterConfig, ClusterModel

            cluster = ClusterModel(model, ClusterConfig(tp_size=1, pp_size=1, dp_size=world,
                                                        use_ddp=True))
            model = cluster.model
            mode = ("reference has no expert parallelism: ClusterModel(dp_size=N, use_ddp=True) "
                    "(fp32 params + bf16 autocast), every expert on every rank")
        else:
            mode = "single device (fp32 params + bf16 autocast, reference Trainer default)"
    else:
        if world < 2:
            raise RuntimeError("TR-MHA 7B training needs tensor parallelism over >= 2 GPUs")
        from complexity.parallel.cluster import ClusterConfig, ClusterModel

        model = model.to(torch.bfloat16)
        cluster = ClusterModel(model, ClusterConfig(tp_size=world, pp_size=1, dp_size=1))
        model = cluster.model.to("cuda").to(torch.bfloat16)
        torch.cuda.empty_cache()
        autocast = False
        mode = (f"reference ClusterModel(tp_size={world}): attention sharded, FFN replicated, "
                "bf16 params")
    inner = getattr(model, "module", model)
    head = inner.lm_head if getattr(inner, "lm_head", None) is not None else inner.embed_tokens
    decay = [p for n, p in model.named_parameters() if "norm" not in n and "bias" not in n]
    nodecay = [p for n, p in model.named_parameters() if "norm" in n or "bias" in n]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1},
                             {"params": nodecay, "weight_decay": 0.0}], lr=3e-4,
                            betas=(0.9, 0.95), foreach=False)

    def step(ids, sync):
        ids = ids.to("cuda", non_blocking=True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            out = model(ids, return_logits=False)
            hidden = out["last_hidden_state"][:, :-1, :].contiguous()
            loss, _ = fused_linear_causal_lm_loss(hidden, head.weight, ids[:, 1:].contiguous(),
                                                  sync_metrics=False)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return float(loss.detach()) if sync else loss.detach()

    return step, mode


def main(args, world, rank, local, helpers):
    """Run ``args.workload``; ``helpers`` is the bench module (timing, clocks,
    Zipf batches, launch counting)."""
    import torch.distributed as dist

    spec = SPEC[args.workload]
    B, S, V = spec["batch"], spec["seq"], spec["arch"]["vocab_size"]
    try:
        build = build_ours if args.impl == "ours" else build_reference
        step, mode = build(args.workload, world)
    except Exception as exc:
        if rank == 0:
            line = {"metric": spec["metric"], "n_gpus": world,
                    "unavailable": f"{type(exc).__name__}: "
                                   f"{str(exc).splitlines()[0] if str(exc) else ''}"}
            if args.impl == "reference":
                line["impl"] = "reference"
            print(json.dumps(line))
        if args.impl == "reference" or isinstance(exc, RuntimeError):
            return
        raise
    if spec["zipf"]:
        host = helpers.zipf_batches(4, B, S, V, seed=1234 + rank)
    else:  # tensor parallel: every rank of the group trains on the same batch
        host = _uniform(4, B, S, V, seed=1234)
    dev = [h.to("cuda") for h in host]
    for i in range(args.warmup):
        step(dev[i % 4], False)
    torch.cuda.synchronize()

    clocks = helpers.ClockSampler(local)
    if local == 0:
        clocks.start()
    ms = helpers.timed(lambda i: step(dev[i % 4], False), args.steps, world)
    clk = clocks.stop() if local == 0 else None

    data_ranks = world if args.workload == "ep1b" else 1
    tokens = B * S * data_ranks
    e2e = None
    if not args.no_e2e:
        k2 = args.e2e_steps or args.steps
        t0 = time.perf_counter()
        ms_e2e = helpers.timed(lambda i: step(host[i % 4], True), k2, world)
        wall = (time.perf_counter() - t0) / k2 * 1000
        e2e = {"value": tokens / (ms_e2e / 1000.0), "unit": "tokens/s", "ms_per_step": ms_e2e,
               "wall_ms_per_step": wall,
               "h2d_bytes_per_step": host[0].numel() * host[0].element_size(),
               "d2h_bytes_per_step": 4,
               "api": ("complexity_framework_b200.training.Trainer.train_step"
                       if args.impl == "ours" else "reference model + fused_linear_causal_lm_loss")}
    launches = None
    if args.impl == "ours" and not args.no_count:
        ours, total = helpers.count_our_kernels(step, dev[0])
        launches = (ours * args.steps, total * args.steps)
    value = tokens / (ms / 1000.0)
    if rank == 0:
        par = (f"ep{world}+dp{world}" if args.workload == "ep1b" and world > 1 else
               f"tp{world}" if args.workload == "tp7b" else "dp1")
        line = {
            "metric": spec["metric"], "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": spec["scaling"], "vs_baseline": None,
            "dtype": "bf16",
            "data": ("synthetic Zipf(1.1) token ids" if spec["zipf"] else
                     "synthetic uniform random token ids") + ", random-init weights",
            "config": {"model": spec["model"], "global_batch": B * data_ranks,
                       "micro_batch_per_gpu": B if data_ranks > 1 or world == 1 else None,
                       "seq_len": S, "parallelism": par, "mode": mode,
                       "l2": "activations larger than L2 (no flush needed)"},
            "clocks": clk, "e2e": e2e,
        }
        if args.impl == "ours":
            if launches is not None:
                line["gpu_launches"], line["gpu_launches_all"] = launches
        else:
            line["impl"] = "reference"
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
