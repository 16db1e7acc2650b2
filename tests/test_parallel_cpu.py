"""Multi-process (gloo, CPU) checks of tensor, pipeline, expert and ZeRO-2 data parallelism.

Every parallel run is compared with a single-process run of the same model,
weights and data.
"""
import copy
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from complexity_framework_b200 import ComplexityModel, ModelConfig

CFG = dict(hidden_size=64, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
           vocab_size=256, intermediate_size=128, shared_intermediate_size=128, num_experts=4,
           top_k=2, routing_strategy="token_id_multi_hash", max_position_embeddings=64)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(world, fn, *args):
    port = _port()
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_entry, args=(r, world, port, fn, d) + args)
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(180)
        codes = [p.exitcode for p in procs]
        assert all(c == 0 for c in codes), codes


def _entry(rank, world, port, fn, tmp, *args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    try:
        fn(rank, world, tmp, *args)
    finally:
        dist.destroy_process_group()


def _model():
    torch.manual_seed(0)
    return ComplexityModel(ModelConfig(**CFG))


def _ids(n=2, s=16, seed=1):
    return torch.randint(0, 256, (n, s), generator=torch.Generator().manual_seed(seed))


def _tp_body(rank, world, tmp):
    from complexity_framework_b200.parallel import gather_tp_state_dict, make_parallel

    ref = _model()
    ids = _ids()
    l_ref = ref.loss(ids)
    l_ref.backward()
    m = make_parallel(_model(), dist.group.WORLD)
    loss = m.loss(ids)
    loss.backward()
    assert torch.allclose(loss, l_ref, atol=1e-5), (loss, l_ref)
    # gradient of a sharded weight matches the matching slice of the full gradient
    a_ref = ref.layers[1].self_attn.q_proj.weight.grad
    a = m.layers[1].self_attn.q_proj.weight.grad
    rows = a.shape[0]
    assert torch.allclose(a, a_ref[rank * rows:(rank + 1) * rows], atol=1e-5)
    e_ref = ref.layers[0].mlp.engine.expert_down.grad
    e = m.layers[0].mlp.engine.expert_down.grad
    w = e.shape[1]
    assert torch.allclose(e, e_ref[:, rank * w:(rank + 1) * w], atol=1e-5)
    # replicated embedding grads are complete on every rank (input-grad all-reduce works)
    assert torch.allclose(m.embed_tokens.weight.grad, ref.embed_tokens.weight.grad, atol=1e-5)
    full = gather_tp_state_dict(m)
    for k, v in ref.state_dict().items():
        assert torch.allclose(full[k].float(), v.float()), k


def test_tensor_parallel_matches_single():
    _run(2, _tp_body)


def _tp_decode_body(rank, world, tmp):
    """Tensor-parallel paged decoding (uneven 128-column shared blocks) gives the
    single-process engine's greedy tokens; the sharded weights gather back."""
    from complexity_framework_b200.inference.engine import (GenerationConfig, InferenceConfig,
                                                            InferenceEngine)
    from complexity_framework_b200.parallel import gather_tp_state_dict
    from complexity_framework_b200.parallel.tp_inference import enable_tp_decode

    cfg = dict(CFG, hidden_size=64, shared_intermediate_size=384, intermediate_size=64)

    def model():
        torch.manual_seed(0)
        return ComplexityModel(ModelConfig(**cfg)).eval()

    prompts = [torch.randint(0, 256, (n,), generator=torch.Generator().manual_seed(n)).tolist()
               for n in (5, 11, 3)]
    gen = GenerationConfig(max_new_tokens=6)
    want = InferenceEngine(model(), InferenceConfig(max_cache_length=64)).generate_tokens(
        prompts, gen)
    ref_state = model().state_dict()
    m = enable_tp_decode(model(), dist.group.WORLD)
    eng = m.layers[0].mlp.engine
    # 384 = 3 blocks of 128 over 2 ranks: rank 0 holds 256 columns, rank 1 holds 128
    assert eng.config.shared_width == (256 if rank == 0 else 128)
    got = InferenceEngine(m, InferenceConfig(max_cache_length=64)).generate_tokens(prompts, gen)
    assert got == want, (got, want)
    full = gather_tp_state_dict(m)
    for k, v in ref_state.items():
        assert torch.allclose(full[k].float(), v.float()), k


def test_tensor_parallel_decode_matches_single():
    _run(2, _tp_decode_body)


def _pp_body(rank, world, tmp, schedule):
    from complexity_framework_b200.parallel import PipelineModel

    ref = _model()
    ids = _ids(4)
    mbs = list(ids.chunk(4))
    l_ref = sum(ref.loss(mb) for mb in mbs) / 4
    l_ref.backward()
    pm = PipelineModel(_model(), schedule=schedule)
    loss = pm.train_step(mbs)
    if pm.last:
        assert torch.allclose(loss, l_ref, atol=1e-5), (loss, l_ref)
    for layer in pm.stage.layers:
        g = layer.self_attn.o_proj.weight.grad
        g_ref = ref.layers[layer.layer_idx].self_attn.o_proj.weight.grad
        assert torch.allclose(g, g_ref, atol=1e-5)
    tied = pm.stage.embed_tokens.weight.grad if pm.first else pm.stage.head_weight.grad
    assert torch.allclose(tied, ref.embed_tokens.weight.grad, atol=1e-5)


@pytest.mark.parametrize("schedule", ["1f1b", "gpipe"])
def test_pipeline_matches_single(schedule):
    _run(2, _pp_body, schedule)


def _ep_body(rank, world, tmp):
    from complexity_framework_b200.parallel import make_expert_parallel

    ref = _model()
    ids_all = _ids(4, seed=3)
    l_ref = ref.loss(ids_all)
    l_ref.backward()
    m = make_expert_parallel(_model(), dist.group.WORLD)
    ids = ids_all.chunk(world)[rank]
    loss = m.loss(ids)
    (loss / world).backward()
    t = loss.detach().clone()
    dist.all_reduce(t)
    assert torch.allclose(t / world, l_ref, atol=1e-5)
    ep = m.layers[2].mlp.engine.ep
    g_ref = ref.layers[2].mlp.engine.expert_gate.grad[ep.lo:ep.lo + ep.E_local]
    assert torch.allclose(ep.expert_gate.grad, g_ref, atol=1e-5)


def test_expert_parallel_matches_single():
    _run(2, _ep_body)


def _ep_trainer_body(rank, world, tmp, mode):
    """Trainer over an expert-parallel model: replicated parameters averaged over
    ranks, expert shards kept rank-local (not overwritten by the start-up
    broadcast) and averaged by 1/world; three AdamW steps with clipping equal
    one process on the whole batch."""
    from complexity_framework_b200.parallel import make_expert_parallel
    from complexity_framework_b200.training import Trainer, TrainingConfig

    ids_all = _ids(4, seed=11)
    cfg = TrainingConfig(learning_rate=1e-3, warmup_steps=0, lr_scheduler="constant",
                         precision="fp32", grad_clip=0.5, distributed_mode=mode,
                         checkpoint_dir=tmp)
    single = Trainer(_model(), cfg, device="cpu", process_group=dist.new_group([rank]))
    for _ in range(3):
        single.train_step(ids_all)
    tr = Trainer(make_expert_parallel(_model(), dist.group.WORLD), cfg, device="cpu")
    for _ in range(3):
        tr.train_step(ids_all.chunk(world)[rank])
    want = dict(single.model.named_parameters())
    for n, p in tr.model.named_parameters():
        if ".ep." in n:
            ep = tr.model.layers[int(n.split(".")[1])].mlp.engine.ep
            full = want[n.replace(".ep.", ".")][ep.lo:ep.lo + ep.E_local]
            assert torch.allclose(p, full, atol=2e-5), n
        else:
            assert torch.allclose(p, want[n], atol=2e-5), n


@pytest.mark.parametrize("mode", ["ddp", "fsdp"])
def test_expert_parallel_trainer_matches_single(mode):
    _run(2, _ep_trainer_body, mode)


def _zero_body(rank, world, tmp, mode):
    from complexity_framework_b200.training import Trainer, TrainingConfig

    ids_all = _ids(4, seed=7)
    cfg = TrainingConfig(learning_rate=1e-3, warmup_steps=0, lr_scheduler="constant",
                         precision="fp32", distributed_mode=mode, checkpoint_dir=tmp)
    single = Trainer(_model(), cfg, device="cpu", process_group=dist.new_group([rank]))
    for _ in range(3):
        single.train_step(ids_all)
    tr = Trainer(_model(), cfg, device="cpu")
    for _ in range(3):
        tr.train_step(ids_all.chunk(world)[rank])
    for (n, p), q in zip(tr.model.named_parameters(), single.model.parameters()):
        assert torch.allclose(p, q, atol=2e-5), n


@pytest.mark.parametrize("mode", ["ddp", "fsdp"])
def test_data_parallel_matches_single(mode):
    _run(2, _zero_body, mode)


def _export_pp_body(rank, world, tmp):
    """Export-traced pipe (torch.distributed.pipelining), 2 stages x 2 microbatches,
    1F1B: the last stage's loss and a first-stage gradient match one process."""
    from complexity_framework_b200.parallel.pipeline_export import (ExportPipelineRunner,
                                                                      trace_pipeline)

    def loss_fn(hidden, labels):
        logits = hidden @ ref.embed_tokens.weight.detach().t()
        return torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)),
                                                 labels.reshape(-1))

    ref = _model()
    ids = _ids(n=4, s=16)
    labels = torch.roll(ids, -1, 1)
    # single process: the same model, head weight treated as a constant
    hidden = ref(ids, return_logits=False)["last_hidden_state"]
    full = 0.5 * (loss_fn(hidden[:2], labels[:2]) + loss_fn(hidden[2:], labels[2:]))
    full.backward()
    want_grad = ref.layers[0].self_attn.o_proj.weight.grad.clone()

    model = _model()
    pipe = trace_pipeline(model, ids[:2], pp_size=world)
    runner = ExportPipelineRunner(pipe, rank, world, torch.device("cpu"), n_microbatches=2,
                                  loss_fn=loss_fn, schedule="1f1b")
    out = runner.step(ids if rank == 0 else None, labels if rank == world - 1 else None)
    if rank == world - 1:
        assert torch.allclose(out, full.detach(), atol=1e-5), (out, full)
    if rank == 0:
        g = dict(runner.module.named_parameters())
        name = next(n for n in g if n.endswith("layers.0.self_attn.o_proj.weight"))
        # the schedule scales each microbatch's loss by 1 / n_microbatches, so the
        # accumulated gradient is that of the mean over microbatches
        assert torch.allclose(g[name].grad, want_grad, atol=1e-6)


def test_export_pipeline_two_stages_match_single_process():
    _run(2, _export_pp_body)


def test_export_pipeline_split_spec():
    from torch.distributed.pipelining import SplitPoint

    from complexity_framework_b200.parallel.pipeline_export import pipeline_split_spec

    assert pipeline_split_spec(32, 8) == {f"layers.{i}": SplitPoint.BEGINNING
                                          for i in range(4, 32, 4)}
    with pytest.raises(ValueError, match="divisible"):
        pipeline_split_spec(30, 8)
    assert pipeline_split_spec(30, 8, require_even=False)["layers.3"] is SplitPoint.BEGINNING


def _zero3_body(rank, world, tmp):
    """ZeRO-3 (parameters, gradient owners and optimizer state sharded per block)
    trains like one process on the same global batch; checkpoints gather."""
    from complexity_framework_b200.training import Trainer, TrainingConfig

    ids = _ids(4, 16, seed=5)
    local = ids.chunk(world)[rank]
    cfg = dict(learning_rate=1e-2, warmup_steps=0, lr_scheduler="constant", grad_clip=1.0,
               skip_param_update_check=False, precision="fp32", max_steps=100,
               checkpoint_dir=os.path.join(tmp, "ck"))
    ref = Trainer(_model(), TrainingConfig(**dict(cfg, distributed_mode="none",
                                                  checkpoint_dir=os.path.join(tmp, "ref"))),
                  process_group=None)
    # one-process reference on the full batch (loss = mean over both halves)
    ref.world = 1
    tr = Trainer(_model(), TrainingConfig(**dict(cfg, distributed_mode="zero3")))
    assert tr.zero3 is not None and tr.distributed_mode == "zero3"
    u0 = tr.zero3.units[0]
    assert u0.shard * world == u0.numel and u0.master.numel() == u0.shard
    for _ in range(3):
        l_ref = ref._train_step_eager(ids, sync=True)
        l = tr.train_step(local, sync=True)
    full = tr.zero3.full_state_dict()
    want = ref.model.state_dict()
    bad = {k: (full[k].float() - v.float()).abs().max().item() for k, v in want.items()
           if not torch.allclose(full[k].float(), v.float(), atol=1e-4)}
    assert not bad, bad
    tr.save_checkpoint()
    if rank == 0:
        assert os.path.exists(os.path.join(tmp, "ck"))


def test_zero3_matches_single_process():
    _run(2, _zero3_body)


def _helpers_body(rank, world, tmp):
    from complexity_framework_b200.parallel import pipeline_parallel as PP
    from complexity_framework_b200.parallel import tensor_parallel as TP

    TP.init_tensor_parallel_group(world)
    assert TP.get_tensor_parallel_world_size() == world and TP.get_tensor_parallel_rank() == rank
    x = torch.full((2, 4), float(rank + 1), requires_grad=True)
    g = TP.all_gather(x, dim=-1)
    assert g.shape == (2, 4 * world) and torch.equal(g[:, 4:], torch.full((2, 4), 2.0))
    (g * torch.arange(8.0)).sum().backward()  # backward: reduce-scatter of the gradient
    assert torch.allclose(x.grad, world * torch.arange(8.0)[rank * 4:(rank + 1) * 4].expand(2, 4))
    y = torch.arange(8.0).repeat(2, 1) * (rank + 1)
    rs = TP.reduce_scatter(y, dim=-1)
    assert torch.equal(rs, 3 * torch.arange(8.0)[rank * 4:(rank + 1) * 4].repeat(2, 1))
    assert torch.equal(TP.all_reduce(torch.ones(3)), torch.full((3,), float(world)))
    if rank == 0:
        PP.send_forward(torch.arange(6.0).view(2, 3), 1)
        got = PP.recv_backward((2, 3), torch.float32, 1, "cpu")
        assert torch.equal(got, -torch.arange(6.0).view(2, 3))
    else:
        got = PP.recv_forward((2, 3), torch.float32, 0, "cpu")
        PP.send_backward(-got, 0)
    assert PP.get_pipeline_parallel_world_size() == world


def test_reference_helper_names_gloo():
    _run(2, _helpers_body)
