"""Fused NVLink data-parallel reduce + AdamW kernels.

* single GPU: a peer that never signals makes the bounded device wait expire;
  the kernel records the error and returns (the context stays usable).
* two GPUs: fused training equals the NCCL reduce-scatter / all-gather path.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def test_peer_timeout_reports_error():
    from complexity_framework_b200.ops import require

    C = require()
    n = 1024
    grad = torch.zeros(n, device="cuda", dtype=torch.bfloat16)
    param = torch.zeros(n, device="cuda", dtype=torch.bfloat16)
    pads = [torch.zeros(64, device="cuda", dtype=torch.int32) for _ in range(2)]
    gs = torch.empty(n // 2, device="cuda", dtype=torch.bfloat16)
    sumsq = torch.zeros(1, device="cuda")
    ticket = torch.zeros(1, device="cuda", dtype=torch.int32)
    ptr = [grad.data_ptr(), grad.data_ptr()]
    pp = [param.data_ptr(), param.data_ptr()]
    pad = [pads[0].data_ptr(), pads[1].data_ptr()]
    slots = [p + 96 for p in pad]
    err = C.error_buffer(0)
    err.zero_()
    # rank 0 of a 2-rank group whose peer never arrives: pads[0][1] stays 0
    C.dp_reduce_shard(ptr, pp, pad, slots, 0, 0, n // 2, gs, sumsq, ticket, 1, True)
    torch.cuda.synchronize()
    vals = err.cpu().tolist()
    assert vals[0] == 5, vals  # kErrPeerTimeout
    err.zero_()
    x = torch.ones(4, device="cuda") * 2  # context still usable
    assert x.sum().item() == 8


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _body(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.training import Trainer, TrainingConfig

    cfg = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
               vocab_size=2048, intermediate_size=256, shared_intermediate_size=512,
               num_experts=4, top_k=2, max_position_embeddings=256)
    ids = torch.randint(0, 2048, (4, 128), generator=torch.Generator().manual_seed(rank))
    res = []
    for fused in ("1", "0"):
        os.environ["CFB_FUSED_DP"] = fused
        torch.manual_seed(0)
        tr = Trainer(ComplexityModel(ModelConfig(**cfg)),
                     TrainingConfig(learning_rate=1e-3, warmup_steps=0, lr_scheduler="constant",
                                    distributed_mode="fsdp", skip_param_update_check=True))
        assert (tr.optimizer._fused is not None) == (fused == "1")
        for _ in range(3):
            tr.train_step(ids)
        res.append(torch.cat([p.detach().float().reshape(-1) for p in tr.model.parameters()]))
    from complexity_framework_b200.ops import check_errors

    torch.cuda.synchronize()
    check_errors(rank)
    diff = (res[0] - res[1]).abs().max().item()
    q.put((rank, diff))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_dp_matches_nccl_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_body, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    diffs = dict(q.get() for _ in range(2))
    assert max(diffs.values()) < 2e-2, diffs


def _graph_body(rank, world, port, q):
    """Fused NVLink data parallel: the replayed CUDA-graph step equals the eager
    step (device barrier epochs and device lr / bias corrections across replays)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), CFB_FUSED_DP="1")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.training import Trainer, TrainingConfig

    cfg = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
               vocab_size=2048, intermediate_size=256, shared_intermediate_size=512,
               num_experts=4, top_k=2, max_position_embeddings=256)
    batches = [torch.randint(0, 2048, (4, 128), generator=torch.Generator().manual_seed(10 * rank + i))
               for i in range(6)]
    res = []
    for graph in (False, True):
        torch.manual_seed(0)
        tr = Trainer(ComplexityModel(ModelConfig(**cfg)),
                     TrainingConfig(learning_rate=1e-3, warmup_steps=2, lr_scheduler="cosine",
                                    max_steps=6, grad_clip=1.0, distributed_mode="fsdp",
                                    skip_param_update_check=True, cuda_graph=graph,
                                    cuda_graph_warmup=2))
        assert tr.optimizer._fused is not None
        for b in batches:
            tr.train_step(b)
        if graph:
            assert tr._graphed is not None and tr._graphed.graph is not None
        res.append(torch.cat([p.detach().float().reshape(-1) for p in tr.model.parameters()]))
    torch.cuda.synchronize()
    check_errors(rank)
    q.put((rank, (res[0] - res[1]).abs().max().item()))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_dp_graph_replay_matches_eager_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_graph_body, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    diffs = dict(q.get() for _ in range(2))
    assert max(diffs.values()) < 1e-2, diffs


def _zero3_body(rank, world, port, q):
    """ZeRO-3 over NVLink (per-block shards, gathers one block ahead, gradient
    reduce-scatter during backward) trains like the ZeRO-2 fused path."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.training import Trainer, TrainingConfig

    cfg = dict(hidden_size=256, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
               vocab_size=2048, intermediate_size=256, shared_intermediate_size=512,
               num_experts=4, top_k=2, max_position_embeddings=256)
    batches = [torch.randint(0, 2048, (4, 128), generator=torch.Generator().manual_seed(10 * rank + i))
               for i in range(4)]
    res, losses = [], []
    for mode in ("fsdp", "zero3"):
        torch.manual_seed(0)
        tr = Trainer(ComplexityModel(ModelConfig(**cfg)),
                     TrainingConfig(learning_rate=1e-3, warmup_steps=0, lr_scheduler="constant",
                                    grad_clip=1.0, distributed_mode=mode,
                                    skip_param_update_check=False))
        assert (tr.zero3 is not None) == (mode == "zero3")
        if tr.zero3 is not None:
            assert tr.zero3.fused
        ls = [tr.train_step(b) for b in batches]
        losses.append(ls)
        if tr.zero3 is not None:
            sd = tr.zero3.full_state_dict()
            res.append(torch.cat([sd[n].float().reshape(-1) for n, _ in
                                  tr.model.named_parameters()]))
        else:
            res.append(torch.cat([p.detach().float().reshape(-1) for p in tr.model.parameters()]))
    torch.cuda.synchronize()
    check_errors(rank)
    q.put((rank, (res[0] - res[1]).abs().max().item(),
           max(abs(a - b) for a, b in zip(*losses))))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero3_matches_zero2_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_zero3_body, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict((r, (d, l)) for r, d, l in (q.get() for _ in range(2)))
    for r, (d, l) in res.items():
        assert d < 2e-2 and l < 2e-2, (r, d, l)
