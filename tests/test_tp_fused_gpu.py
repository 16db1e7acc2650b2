"""Fused tensor-parallel GEMMs on 2 GPUs: the all-gather runs inside the GEMM
(copier warps pull peer row chunks over NVLink into the local gathered operand,
which the TMA producer then reads), the reduce-scatter writes local bf16
partials that a finish kernel sums by reading the owned rows of every peer.
Forward and backward are compared with the same math on one GPU in fp32."""
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
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.parallel.tp_fused import TPWorkspace, ag_linear, rs_linear

    torch.manual_seed(0)
    T, H, F = 1024, 256, 512  # tokens, hidden, ffn (split over ranks)
    x = torch.randn(T, H, device="cuda") * 0.5
    w1 = torch.randn(F, H, device="cuda") / H ** 0.5      # column parallel
    w2 = torch.randn(H, F, device="cuda") / F ** 0.5      # row parallel
    res = torch.randn(T, H, device="cuda")
    gout = torch.randn(T, H, device="cuda")
    rows = T // world
    sl = slice(rank * rows, (rank + 1) * rows)
    fl = slice(rank * F // world, (rank + 1) * F // world)

    # reference (fp32, one GPU, full tensors)
    xr = x.clone().requires_grad_()
    w1r = w1.clone().requires_grad_()
    w2r = w2.clone().requires_grad_()
    hr = xr.bfloat16().float() @ w1r.bfloat16().float().t()
    outr = hr.bfloat16().float() @ w2r.bfloat16().float().t() + res.bfloat16().float()
    (outr * gout).sum().backward()

    ws = TPWorkspace()
    ws.begin_step()
    xs = x[sl].bfloat16().contiguous().requires_grad_()
    w1s = w1[fl].bfloat16().contiguous().requires_grad_()
    w2s = w2[:, fl].bfloat16().contiguous().requires_grad_()
    h = ag_linear(xs, w1s, ws, "l0.fc1")                       # [T, F/P]
    out = rs_linear(h, w2s, res[sl].bfloat16(), ws, "l0.fc2")  # [T/P, H]
    (out.float() * gout[sl]).sum().backward()
    torch.cuda.synchronize()
    check_errors(rank)

    def rel(a, b):
        return float((a.float() - b).abs().max() / b.abs().max().clamp_min(1e-6))

    errs = {"h": rel(h, hr[:, fl]), "out": rel(out, outr[sl]), "dx": rel(xs.grad, xr.grad[sl]),
            "dw1": rel(w1s.grad, w1r.grad[fl]), "dw2": rel(w2s.grad, w2r.grad[:, fl])}
    q.put((rank, errs))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_tp_ag_rs_two_gpus():
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
        assert max(errs.values()) < 3e-2, (r, errs)


def _model_body(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    import copy

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.parallel.tp_fused import (allreduce_replicated_grads,
                                                             enable_fused_sequence_parallel)

    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=2048, intermediate_size=256,
                      shared_intermediate_size=512, num_experts=4, top_k=2,
                      routing_strategy="token_id_multi_hash", max_position_embeddings=256)
    torch.manual_seed(0)
    ref = ComplexityModel(cfg).cuda().bfloat16().train()
    ids = torch.randint(0, 2048, (2, 256), generator=torch.Generator().manual_seed(1)).cuda()
    loss_ref = ref.loss(ids)
    loss_ref.backward()
    sp = enable_fused_sequence_parallel(copy.deepcopy(ref).train())
    for p in sp.parameters():
        p.grad = None
    share = sp.loss(ids)
    share.backward()
    allreduce_replicated_grads(sp)
    tot = share.detach().float().clone()
    dist.all_reduce(tot)
    torch.cuda.synchronize()
    check_errors(rank)
    g_ref = dict(ref.named_parameters())

    def rel(a, b):
        return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))

    errs = {"loss": abs(float(tot) - float(loss_ref)) / float(loss_ref)}
    for name, p in sp.named_parameters():
        if p.grad is None:
            continue
        full = g_ref[name].grad
        if hasattr(p, "_tp_shard_dim"):
            d = p._tp_shard_dim
            n = p.shape[d]
            full = full.narrow(d, rank * n, n)
        errs[name] = rel(p.grad, full)
    q.put((rank, errs))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_sequence_parallel_model_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_model_body, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    out = dict(q.get() for _ in range(2))
    for r, errs in out.items():
        assert errs["loss"] < 1e-2, (r, errs["loss"])
        bad = {k: round(v, 4) for k, v in errs.items() if v >= 6e-2}
        assert not bad, (r, bad)


def _trainer_body(rank, world, port, q, shared=512):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    import copy

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.parallel.tp_fused import enable_fused_sequence_parallel
    from complexity_framework_b200.training import Trainer, TrainingConfig

    cfg = ModelConfig(hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=2048, intermediate_size=256,
                      shared_intermediate_size=shared, num_experts=4, top_k=2,
                      routing_strategy="token_id_multi_hash", max_position_embeddings=256)
    tc = dict(learning_rate=2e-3, warmup_steps=0, lr_scheduler="constant",
              skip_param_update_check=True)
    ids = torch.randint(0, 2048, (2, 256), generator=torch.Generator().manual_seed(3))
    torch.manual_seed(0)
    base = ComplexityModel(cfg)
    sp = enable_fused_sequence_parallel(copy.deepcopy(base).cuda().bfloat16())
    tr_sp = Trainer(sp, TrainingConfig(**tc))
    losses_sp = [tr_sp.train_step(ids) for _ in range(4)]
    torch.cuda.synchronize()
    check_errors(rank)
    losses_ref = None
    from complexity_framework_b200.training.trainer import _singleton_group

    solo = _singleton_group(dist.group.WORLD)  # collective
    if rank == 0:
        # single-GPU reference run (no process group involvement)
        ref_model = copy.deepcopy(base).cuda().bfloat16()
        from complexity_framework_b200.training.optim import FusedAdamW, default_param_groups

        opt = FusedAdamW(default_param_groups(ref_model, 0.1), lr=2e-3, betas=(0.9, 0.95),
                         weight_decay=0.1, process_group=solo)
        losses_ref = []
        for _ in range(4):
            loss = ref_model.loss(ids.cuda())
            loss.backward()
            opt.reduce_gradients()
            opt.clip_grad_norm_(1.0)
            opt.step(clip=True)
            opt.zero_grad()
            losses_ref.append(float(loss))
    q.put((rank, losses_sp, losses_ref))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("shared", [512, 384])  # 384 / 2 = 192: shard padded to 256
def test_trainer_fused_sequence_parallel_two_gpus(shared):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_trainer_body, args=(r, 2, port, q, shared)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = {r: (a, b) for r, a, b in (q.get() for _ in range(2))}
    sp0, ref = res[0]
    sp1, _ = res[1]
    assert sp0 == sp1  # every TP rank reports the same global loss
    assert sp0[-1] < sp0[0]
    for a, b in zip(sp0, ref):
        assert abs(a - b) / b < 2e-2, (sp0, ref)
