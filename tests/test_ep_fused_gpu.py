"""Expert parallelism with NVLink dispatch/combine kernels on 2 GPUs vs one GPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _body(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    import copy

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.parallel.ep_fused import make_fused_expert_parallel

    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=2048, intermediate_size=512,
                      shared_intermediate_size=512, num_experts=4, top_k=2,
                      routing_strategy="token_id_multi_hash", max_position_embeddings=256)
    torch.manual_seed(0)
    ref = ComplexityModel(cfg).cuda().bfloat16().train()
    ids = torch.randint(0, 2048, (2, 256), generator=torch.Generator().manual_seed(5)).cuda()
    loss_ref = ref.loss(ids)
    loss_ref.backward()
    ep = make_fused_expert_parallel(copy.deepcopy(ref).train())
    for p in ep.parameters():
        p.grad = None
    loss = ep.loss(ids)  # both ranks see the same tokens
    loss.backward()
    torch.cuda.synchronize()
    check_errors(rank)
    g_ref = dict(ref.named_parameters())

    def rel(a, b):
        return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))

    errs = {"loss": abs(float(loss) - float(loss_ref)) / float(loss_ref)}
    El = 2
    for name, p in ep.named_parameters():
        if p.grad is None:
            continue
        if ".ep.expert_" in name:
            full = g_ref[name.replace(".ep.", ".")].grad[rank * El:(rank + 1) * El]
            errs[name] = rel(p.grad / world, full)  # every rank contributed its (equal) tokens
        else:
            errs[name] = rel(p.grad, g_ref[name].grad)
    q.put((rank, errs))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_expert_parallel_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_body, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    out = dict(q.get() for _ in range(2))
    for r, errs in out.items():
        assert errs["loss"] < 5e-3, (r, errs["loss"])
        bad = {k: round(v, 4) for k, v in errs.items() if v >= 6e-2}
        assert not bad, (r, bad)
