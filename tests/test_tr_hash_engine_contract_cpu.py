"""Contract surfaces of the TR-Hash engine that manifests and user code rely on.

Runtime capacity (``set_active_capacity``), exact route-table installation
(``load_route_table``), the backend decision matrix (``select_backend``) and
the ``capability_summary`` key set.  Counterparts: tests/test_tr_hash_engine.py
and tests/test_tr_hash_dynamic_moe.py of the reference, covering the behaviour
of complexity/tr_hash/engine.py and complexity/tr_hash/capabilities.py.
"""
import pytest
import torch

from complexity_framework_b200.tr_hash import (AttentionBackbone, GraphBucket, TRHashBackend,
                                               TRHashEngine, TRHashEngineConfig, TRHashPhase,
                                               TRHashPrecision, TRHashStrategy, build_route_table,
                                               select_backend)

SUMMARY_KEYS = {
    "experts", "top_k", "shared_width", "expert_width", "stored_width", "active_width",
    "active_width_fraction", "active_num_experts", "active_expert_width", "is_reduced_capacity",
    "attention", "routing", "phase", "precision", "world_size", "parallelism",
    "requested_backend", "selected_backend", "backend_reasons", "fused_cuda_eligible",
    "cuda_graph_buckets",
}


def _engine(**over):
    kw = dict(hidden_size=16, vocab_size=97, num_experts=8, top_k=2, shared_width=8,
              expert_width=12, routing_strategy=TRHashStrategy.BALANCED_HASH,
              attention_backbone=AttentionBackbone.GQA, phase=TRHashPhase.TRAINING,
              precision=TRHashPrecision.FP32, backend=TRHashBackend.PYTORCH)
    kw.update(over)
    torch.manual_seed(0)
    return TRHashEngine(TRHashEngineConfig(**kw))


def _inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(2, 5, 16, generator=g), torch.randint(0, 97, (2, 5), generator=g)


# ------------------------------------------------------------ capacity
def test_full_capacity_by_default_and_summary_keys():
    e = _engine()
    assert (e.active_num_experts, e.active_expert_width) == (8, 12)
    s = e.capability_summary()
    assert set(s) == SUMMARY_KEYS
    assert s["is_reduced_capacity"] is False
    assert (s["active_num_experts"], s["active_expert_width"]) == (8, 12)


def test_reduced_expert_count_routes_only_into_the_active_pool():
    e = _engine()
    e.set_active_capacity(num_experts=4)
    assert e.is_reduced_capacity and e.capability_summary()["active_num_experts"] == 4
    active = e._active_route_table
    assert 0 <= int(active.min()) and int(active.max()) < 4
    assert int(e.route_table.max()) >= 4                  # the stored table is untouched
    # the reduced table is the builder's table for the smaller pool (pure token-id function)
    sub = TRHashEngineConfig(**{**e.config.__dict__, "num_experts": 4})
    assert torch.equal(active, build_route_table(sub))


def test_reduced_capacity_changes_output_and_full_capacity_restores_it_exactly():
    e = _engine()
    x, ids = _inputs()
    with torch.no_grad():
        full = e(x, ids)
        e.set_active_capacity(num_experts=2)
        fewer = e(x, ids)
        e.set_active_capacity(num_experts=8, expert_width=4)
        narrower = e(x, ids)
        e.set_active_capacity(num_experts=8, expert_width=12)
        again = e(x, ids)
    assert fewer.shape == narrower.shape == full.shape == (2, 5, 16)
    assert not torch.allclose(full, fewer) and not torch.allclose(full, narrower)
    assert torch.equal(full, again)


def test_reduced_width_backward_touches_only_the_active_slice():
    e = _engine()
    e.set_active_capacity(expert_width=4)
    x, ids = _inputs(1)
    e(x.requires_grad_(), ids).square().mean().backward()
    for name in ("expert_gate", "expert_up"):
        g = getattr(e, name).grad
        assert torch.any(g[:, :, :4] != 0) and torch.all(g[:, :, 4:] == 0), name
    g = e.expert_down.grad
    assert torch.any(g[:, :4] != 0) and torch.all(g[:, 4:] == 0)


def test_invalid_capacity_requests_are_rejected():
    e = _engine(num_experts=4)
    for bad in (3, 5, 32):
        with pytest.raises(ValueError, match="must be one of"):
            e.set_active_capacity(num_experts=bad)
    with pytest.raises(ValueError, match="cannot exceed the allocated capacity"):
        e.set_active_capacity(num_experts=8)
    for bad in (0, 13):
        with pytest.raises(ValueError, match="expert_width"):
            e.set_active_capacity(expert_width=bad)


# ------------------------------------------------------- route tables
def test_load_route_table_installs_exact_table_and_pair_metadata():
    e = _engine(num_experts=4, expert_width=8, routing_strategy=TRHashStrategy.MODULO_CYCLIC)
    before_codes = e.fused_route_codes.clone()
    table = torch.stack([torch.arange(97) % 4, (torch.arange(97) + 3) % 4])
    e.load_route_table(table)
    assert torch.equal(e.route_table, table)
    assert torch.equal(e._active_route_table, table)
    assert not torch.equal(e.fused_route_codes, before_codes)     # metadata recompiled
    # a code is the index of the unordered expert pair plus a swap bit (slot 0 holds the
    # larger id); decoding every code gives the installed table back
    pairs = e.fused_expert_pairs.long()
    codes = e.fused_route_codes.long()
    swap_bit = 1 << max(1, (pairs.size(0) - 1).bit_length())
    idx, swap = codes % swap_bit, (codes & swap_bit) != 0
    lo, hi = pairs[idx, 0], pairs[idx, 1]
    decoded = torch.stack([torch.where(swap, hi, lo), torch.where(swap, lo, hi)])
    assert torch.equal(decoded, table)
    with pytest.raises(ValueError, match="does not match"):
        e.load_route_table(table[:, :50])
    with pytest.raises(ValueError, match="out-of-range"):
        e.load_route_table(torch.full((2, 97), 4))


# ------------------------------------------------------- backend choice
def test_backend_decision_matrix():
    def cfg(**over):
        kw = dict(hidden_size=256, vocab_size=101, num_experts=4, top_k=2, shared_width=1024,
                  expert_width=64, precision=TRHashPrecision.BF16)
        kw.update(over)
        return TRHashEngineConfig(**kw)

    cpu = select_backend(cfg(), device_type="cpu")
    assert cpu.selected is TRHashBackend.PYTORCH
    assert "CGGR requires CUDA" in cpu.reasons
    # dense-masked experts when the routed width is cheap, grouped when it is not
    d = select_backend(cfg(), device_type="cuda", cggr_available=True, fused_cuda_available=True)
    assert d.selected is TRHashBackend.FUSED_CUDA
    wide = select_backend(cfg(num_experts=16, expert_width=256), device_type="cuda",
                          cggr_available=True, fused_cuda_available=True)
    assert wide.selected is TRHashBackend.CGGR and wide.reasons
    odd = select_backend(cfg(expert_width=12), device_type="cuda", cggr_available=True,
                         fused_cuda_available=True)
    assert odd.selected is TRHashBackend.CGGR
    # no extension built: reference math, with the reason recorded
    nobuild = select_backend(cfg(), device_type="cuda", cggr_available=True,
                             fused_cuda_available=False)
    assert nobuild.selected is TRHashBackend.PYTORCH and nobuild.reasons
    # explicit requests are honoured or refused, never silently replaced
    with pytest.raises(RuntimeError):
        select_backend(cfg(backend=TRHashBackend.FUSED_CUDA, expert_width=12),
                       device_type="cuda", cggr_available=True, fused_cuda_available=True)
    with pytest.raises(RuntimeError):
        select_backend(cfg(backend=TRHashBackend.CGGR), device_type="cpu")
    assert select_backend(cfg(backend=TRHashBackend.PYTORCH), device_type="cuda",
                          cggr_available=True).selected is TRHashBackend.PYTORCH
    for q in (TRHashPrecision.FP8, TRHashPrecision.INT8):
        with pytest.raises(NotImplementedError):
            select_backend(cfg(precision=q), device_type="cuda", cggr_available=True)


def test_cuda_graph_backend_is_inference_only_with_buckets():
    with pytest.raises(ValueError, match="inference-only"):
        TRHashEngineConfig(hidden_size=8, vocab_size=101, backend=TRHashBackend.CUDA_GRAPH,
                           graph_buckets=(GraphBucket(1, 128),))
    with pytest.raises(ValueError, match="requires at least one"):
        TRHashEngineConfig(hidden_size=8, vocab_size=101, phase=TRHashPhase.INFERENCE,
                           backend=TRHashBackend.CUDA_GRAPH)


def test_auto_under_reduced_capacity_uses_reference_math():
    e = _engine(backend=TRHashBackend.AUTO)
    e.set_active_capacity(num_experts=4)
    d = e.decide("cuda")
    assert d.selected is not TRHashBackend.FUSED_CUDA
    assert e.capability_summary("cpu")["is_reduced_capacity"] is True


@pytest.mark.gpu
def test_reduced_capacity_on_cuda_falls_back_and_matches_pytorch():
    e = _engine(backend=TRHashBackend.AUTO, hidden_size=128, shared_width=256, expert_width=32,
                num_experts=4).cuda()
    ref = _engine(backend=TRHashBackend.PYTORCH, hidden_size=128, shared_width=256,
                  expert_width=32, num_experts=4).cuda()
    ref.load_state_dict(e.state_dict())
    for m in (e, ref):
        m.set_active_capacity(num_experts=2, expert_width=16)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 64, 128, generator=g).cuda()
    ids = torch.randint(0, 97, (2, 64), generator=g).cuda()
    with torch.no_grad():
        out = e(x, ids)
        want = ref(x, ids)
    assert e.last_backend.selected is not TRHashBackend.FUSED_CUDA
    assert torch.allclose(out, want, atol=1e-5)
