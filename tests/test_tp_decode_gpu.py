"""Tensor-parallel paged decoding with the fused NVLink all-reduce (csrc/tp_decode.cu).

* one GPU: a peer that never signals makes the bounded barrier expire; the
  kernel records the error and returns (the context stays usable);
* two GPUs: greedy tokens of graph-replayed decode steps equal the eager
  tensor-parallel engine's, and tensor-parallel prefill logits match the
  unsharded model's.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def test_tp_allreduce_peer_timeout_reports_error():
    from complexity_framework_b200.ops import require

    C = require()
    buf = torch.ones(64, device="cuda", dtype=torch.bfloat16)
    pads = [torch.zeros(32, device="cuda", dtype=torch.int32) for _ in range(2)]
    out = torch.empty(64, device="cuda", dtype=torch.bfloat16)
    epoch = torch.zeros(1, device="cuda", dtype=torch.int32)
    ticket = torch.zeros(1, device="cuda", dtype=torch.int32)
    err = C.error_buffer(0)
    err.zero_()
    # rank 0 of a 2-rank group whose peer never arrives
    C.tp_allreduce([buf.data_ptr()] * 2, [p.data_ptr() for p in pads], 0, 0, None, out,
                   epoch, ticket)
    torch.cuda.synchronize()
    vals = err.cpu().tolist()
    assert vals[0] == 5, vals  # kErrPeerTimeout
    err.zero_()
    assert epoch.item() == 1 and ticket.item() == 0  # epoch advanced, ticket reset
    x = torch.ones(4, device="cuda") * 2
    assert x.sum().item() == 8


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


CFG = dict(hidden_size=512, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
           vocab_size=2048, intermediate_size=512, shared_intermediate_size=1408,
           num_experts=4, top_k=2, routing_strategy="modulo_cyclic", max_position_embeddings=512)


def _body(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.inference.engine import (GenerationConfig, InferenceConfig,
                                                            InferenceEngine, forward_paged)
    from complexity_framework_b200.inference.paged import PagedBatch, PagePool, SeqChunk
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.parallel.tp_inference import enable_tp_decode

    def model():
        torch.manual_seed(0)
        return ComplexityModel(ModelConfig(**CFG)).cuda().to(torch.bfloat16).eval()

    def prefill_logits(m):
        a = m.layers[0].self_attn
        pool = PagePool(len(m.layers), a.num_kv_heads, a.head_dim, 16, 16,
                        dtype=torch.bfloat16, device="cuda")
        pool.allocate_sequence(0)
        ids = torch.randint(0, 2048, (40,), generator=torch.Generator().manual_seed(3)).cuda()
        with torch.no_grad():
            b = PagedBatch(pool, [SeqChunk(0, 0, 40)])
            h = forward_paged(m, ids, b)
            return m.logits(h[None])[0].float()

    ref = prefill_logits(model())
    m = enable_tp_decode(model(), dist.group.WORLD)
    # 1408 = 11 blocks of 128 over 2 ranks: 768 and 640 columns
    assert m.layers[0].mlp.engine.config.shared_width == (768 if rank == 0 else 640)
    got = prefill_logits(m)
    rel = ((got - ref).abs().max() / ref.abs().max()).item()
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, 2048, (int(n),), generator=g).tolist() for n in (9, 30, 17, 64)]
    outs = {}
    for graph in (False, True):
        eng = InferenceEngine(m, InferenceConfig(max_cache_length=512, max_batch_size=8,
                                                 cuda_graph_decode=graph))
        outs[graph] = eng.generate_tokens(prompts, GenerationConfig(max_new_tokens=12))
        if graph:
            assert eng.stats.get("graph_steps", 0) > 0
    torch.cuda.synchronize()
    check_errors(rank)
    q.put((rank, rel, outs[True] == outs[False], m.tp_decode.uses_multicast))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_decode_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_body, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get() for _ in range(2))
    for rank, rel, same, _ in res:
        assert rel < 3e-2, (rank, rel)
        assert same, rank
