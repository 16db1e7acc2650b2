"""Context parallel on B200s (NCCL ranks, one per GPU, up to 2): the fused
attention path with chunk positions and ring / Ulysses attention matches the
full-sequence model on one GPU."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, method, q_out, layout="contiguous"):
    import torch.distributed as dist

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.parallel.context_parallel import (context_parallel_batch,
                                                                      enable_context_parallel)

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    torch.manual_seed(0)
    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=2048, intermediate_size=256,
                      shared_intermediate_size=512, num_experts=4, max_position_embeddings=1024)
    model = ComplexityModel(cfg).cuda().to(torch.bfloat16)
    ids = torch.randint(0, 2048, (2, 512), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        ref = float(model.loss(ids))
        enable_context_parallel(model, None, method, layout)
        x, y = context_parallel_batch(ids, None, layout=layout)
        n_local = (y != -100).sum()
        part = model.loss(x, y) * n_local / (2 * 511)
        dist.all_reduce(part)
    errs = [None] * world
    dist.all_gather_object(errs, abs(float(part) - ref))
    if rank == 0:
        q_out.put(errs)
    dist.destroy_process_group()


@pytest.mark.parametrize("method,layout", [("ring", "contiguous"), ("ulysses", "contiguous"),
                                           ("ring", "zigzag")])
def test_context_parallel_fused_path(method, layout):
    import torch.multiprocessing as mp

    world = min(2, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ps = [ctx.Process(target=_worker, args=(r, world, port, method, q, layout))
          for r in range(world)]
    for p in ps:
        p.start()
    errs = q.get(timeout=240)
    for p in ps:
        p.join(timeout=60)
    assert max(errs) < 3e-2, errs  # bf16 activations, same weights


def test_ring_blocks_on_cudnn_match_sdpa():
    """The ring's block forward / backward on cuDNN flash kernels, merged over
    two causal chunks exactly as the ring merges them, against SDPA."""
    import math

    import torch.nn.functional as F

    from complexity_framework_b200.parallel.context_parallel import (_block_backward,
                                                                      _block_forward,
                                                                      _cudnn_blocks)

    torch.manual_seed(0)
    B, Hq, Hkv, S, D, P = 2, 4, 2, 256, 64, 2
    mk = lambda h: torch.randn(B, h, S, D, device="cuda").bfloat16()  # noqa: E731
    q, k, v, go = mk(Hq), mk(Hkv), mk(Hkv), mk(Hq)
    assert _cudnn_blocks(q)
    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True, enable_gqa=True)
    (ref * go.float()).sum().backward()
    sc = D ** -0.5
    L = S // P
    ch = lambda t, i: t[:, :, i * L:(i + 1) * L]  # noqa: E731
    dk = torch.zeros(B, Hkv, S, D, device="cuda")
    dv = torch.zeros_like(dk)
    for r in range(P):
        lse = torch.full((B, Hq, L, 1), -math.inf, device="cuda")
        acc = torch.zeros(B, Hq, L, D, device="cuda")
        for src in range(r + 1):
            o_b, lse_b = _block_forward(ch(q, r), ch(k, src), ch(v, src), src == r, sc)
            new = torch.logaddexp(lse, lse_b)
            acc = acc * torch.exp(lse - new) + o_b * torch.exp(lse_b - new)
            lse = new
        assert float((acc - ch(ref, r)).abs().max()) < 3e-2
        out = acc.bfloat16()
        dq = torch.zeros(B, Hq, L, D, device="cuda")
        for src in range(r + 1):
            a, b, c = _block_backward(ch(go, r), ch(q, r), ch(k, src), ch(v, src), out, lse,
                                      src == r, sc)
            dq += a
            dk[:, :, src * L:(src + 1) * L] += b
            dv[:, :, src * L:(src + 1) * L] += c
        rel = float((dq - ch(qr.grad, r)).abs().max() / qr.grad.abs().max())
        assert rel < 3e-2, rel
    for got, want in ((dk, kr.grad), (dv, vr.grad)):
        assert float((got - want).abs().max() / want.abs().max()) < 3e-2
