"""Context-parallel attention (ring and Ulysses) on gloo ranks against
single-process attention over the whole sequence: outputs and dq/dk/dv."""
import socket

import pytest
import torch
import torch.nn.functional as F


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, method, causal, q_out, layout="contiguous"):
    import torch.distributed as dist

    from complexity_framework_b200.parallel.context_parallel import (
        context_parallel_attention, split_sequence)

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    g = torch.Generator().manual_seed(0)
    B, Hq, Hkv, S, D = 2, 4, 2, 12, 8
    q = torch.randn(B, Hq, S, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g)
    v = torch.randn(B, Hkv, S, D, generator=g)
    go = torch.randn(B, Hq, S, D, generator=g)
    # reference over the whole sequence
    qr, kr, vr = (t.clone().requires_grad_() for t in (q, k, v))
    o_ref = F.scaled_dot_product_attention(qr, kr, vr, is_causal=causal, enable_gqa=True)
    (o_ref * go).sum().backward()
    # this rank's chunk
    sp = lambda t: split_sequence(t, None, 2, layout)  # noqa: E731
    ql, kl, vl = (sp(t).clone().requires_grad_() for t in (q, k, v))
    o = context_parallel_attention(ql, kl, vl, None, causal=causal, method=method, layout=layout)
    (o * sp(go)).sum().backward()
    err = max(float((o - sp(o_ref)).abs().max()), float((ql.grad - sp(qr.grad)).abs().max()),
              float((kl.grad - sp(kr.grad)).abs().max()),
              float((vl.grad - sp(vr.grad)).abs().max()))
    errs = [None] * world
    dist.all_gather_object(errs, err)
    if rank == 0:
        q_out.put(errs)
    dist.destroy_process_group()


@pytest.mark.parametrize("method,world,layout", [("ring", 3, "contiguous"),
                                                 ("ring", 2, "contiguous"),
                                                 ("ulysses", 2, "contiguous"),
                                                 ("ring", 3, "zigzag")])
@pytest.mark.parametrize("causal", [True, False])
def test_context_parallel_matches_full_attention(method, world, layout, causal):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, method, causal, q, layout))
          for r in range(world)]
    for p in ps:
        p.start()
    errs = q.get(timeout=180)
    for p in ps:
        p.join(timeout=60)
    assert max(errs) < 1e-4, errs


def _model_worker(rank, world, port, method, q_out, layout="contiguous"):
    import torch.distributed as dist

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.parallel.context_parallel import (context_parallel_batch,
                                                                      enable_context_parallel)

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    torch.manual_seed(0)
    cfg = ModelConfig(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=128, intermediate_size=64,
                      shared_intermediate_size=128, num_experts=4, max_position_embeddings=256)
    full = ComplexityModel(cfg)
    ids = torch.randint(0, 128, (2, 32), generator=torch.Generator().manual_seed(3))
    ref_loss = full.loss(ids)
    ref_loss.backward()
    ref_grads = [p.grad.clone() for p in full.parameters()]
    full.zero_grad()
    assert enable_context_parallel(full, None, method, layout) == 2
    x, y = context_parallel_batch(ids, None, layout=layout)
    n_local = (y != -100).sum()
    n_total = (torch.roll(ids, -1, 1)[:, :-1]).numel()
    loss = full.loss(x, y) * n_local / n_total          # this rank's share of the mean
    loss.backward()
    total = loss.detach().clone()
    dist.all_reduce(total)
    err = abs(float(total) - float(ref_loss))
    for p, g in zip(full.parameters(), ref_grads):
        pg = p.grad.contiguous()
        dist.all_reduce(pg)
        err = max(err, float((pg - g).abs().max()))
    errs = [None] * world
    dist.all_gather_object(errs, err)
    if rank == 0:
        q_out.put(errs)
    dist.destroy_process_group()


@pytest.mark.parametrize("method,layout", [("ring", "contiguous"), ("ulysses", "contiguous"),
                                           ("ring", "zigzag")])
def test_model_context_parallel_matches_full_sequence(method, layout):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_model_worker, args=(r, 2, port, method, q, layout))
          for r in range(2)]
    for p in ps:
        p.start()
    errs = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
    assert max(errs) < 1e-4, errs
