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


def _worker(rank, world, port, method, q_out):
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
        enable_context_parallel(model, None, method)
        x, y = context_parallel_batch(ids, None)
        n_local = (y != -100).sum()
        part = model.loss(x, y) * n_local / (2 * 511)
        dist.all_reduce(part)
    errs = [None] * world
    dist.all_gather_object(errs, abs(float(part) - ref))
    if rank == 0:
        q_out.put(errs)
    dist.destroy_process_group()


@pytest.mark.parametrize("method", ["ring", "ulysses"])
def test_context_parallel_fused_path(method):
    import torch.multiprocessing as mp

    world = min(2, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ps = [ctx.Process(target=_worker, args=(r, world, port, method, q)) for r in range(world)]
    for p in ps:
        p.start()
    errs = q.get(timeout=240)
    for p in ps:
        p.join(timeout=60)
    assert max(errs) < 3e-2, errs  # bf16 activations, same weights
