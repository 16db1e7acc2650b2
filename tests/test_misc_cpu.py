"""GPU/runtime helpers, integer ops, safety clamps (CPU parts)."""
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.core.integer_ops import Int8Linear, int8_matmul, lut_silu, quantize_int8_rows
from complexity_framework_b200.utils.gpu import GradientCompressor, clip_grad_norm_fused, dtype_from_string
from complexity_framework_b200.utils.safety import (MultiDirectionSafetyClamp, SafetyClamp,
                                                    get_safety_stats, install_safety,
                                                    remove_safety)


def test_int8_and_lut():
    torch.manual_seed(0)
    lin = torch.nn.Linear(64, 32)
    x = torch.randn(8, 64)
    y = Int8Linear(lin)(x)
    assert float((y - lin(x)).abs().max() / lin(x).abs().max()) < 0.03
    qa, sa = quantize_int8_rows(x)
    qw, sw = quantize_int8_rows(lin.weight.detach())
    assert int8_matmul(qa, sa, qw, sw).shape == (8, 32)
    t = torch.linspace(-6, 6, 100)
    assert float((lut_silu()(t) - torch.nn.functional.silu(t)).abs().max()) < 0.05


def test_clip_and_dtype():
    m = torch.nn.Linear(8, 8)
    m(torch.randn(4, 8)).sum().mul(100).backward()
    ref = torch.nn.utils.get_total_norm([p.grad for p in m.parameters()])
    n = clip_grad_norm_fused(m.parameters(), 1.0)
    assert abs(float(n) - float(ref)) / float(ref) < 1e-5
    assert float(torch.nn.utils.get_total_norm([p.grad for p in m.parameters()])) <= 1.0 + 1e-4
    assert dtype_from_string("bf16") == torch.bfloat16


def _comp(rank, port, method, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    torch.manual_seed(rank)
    m = torch.nn.Linear(16, 16)
    m.weight.grad = torch.full_like(m.weight, float(rank + 1))
    m.bias.grad = torch.zeros_like(m.bias)
    GradientCompressor(method, ratio=1.0).compress_and_allreduce(m)
    q.put((rank, float(m.weight.grad.mean())))
    dist.destroy_process_group()


def test_gradient_compressor_gloo():
    import socket

    for method in ("none", "topk", "quantize"):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
        s.close()
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        ps = [ctx.Process(target=_comp, args=(r, port, method, q)) for r in range(2)]
        [p.start() for p in ps]
        [p.join(120) for p in ps]
        vals = dict(q.get() for _ in range(2))
        assert all(abs(v - 1.5) < 0.02 for v in vals.values()), (method, vals)


def test_safety_clamps():
    d = torch.zeros(8)
    d[0] = 1
    c = SafetyClamp(d, threshold=1.0)
    h = torch.tensor([[5.0] + [0.0] * 7])
    assert float(c(h)[0, 0]) == 1.0
    mc = MultiDirectionSafetyClamp(torch.eye(8)[:2], threshold=0.5)
    assert float(mc(torch.ones(1, 8))[0, :2].max()) <= 0.5 + 1e-5
    m = ComplexityModel(ModelConfig(hidden_size=64, num_hidden_layers=3, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=128, intermediate_size=64,
                                    shared_intermediate_size=128, num_experts=4, top_k=2,
                                    routing_strategy="modulo_cyclic"))
    install_safety(m, torch.randn(64))
    m(torch.randint(0, 128, (1, 8)))
    assert get_safety_stats(m)["calls"] == 1
    remove_safety(m)


def test_integer_ops_reference_names_match_reference():
    import os
    import sys

    import torch

    from complexity_framework_b200.core import integer_ops as I

    ref_root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "baseline", "_ref")
    g = torch.Generator().manual_seed(0)
    w, x = torch.randn(16, 32, generator=g), torch.randn(4, 32, generator=g)
    qw, sw = I.quantize_weight_int8(w)
    y = I.int8_linear(x, qw, sw)
    assert torch.allclose(y, x @ w.t(), atol=0.1, rtol=0.05)
    gg, uu = I.int8_fused_gate_up(x, qw, sw, 8)
    assert gg.shape == (4, 8) and torch.allclose(torch.cat([gg, uu], -1), y)
    z = torch.arange(-1200, 1201, 7, dtype=torch.int32)
    if not os.path.isdir(os.path.join(ref_root, "complexity")):
        return
    sys.path.insert(0, ref_root)
    try:
        from complexity.core import integer_ops as R
    finally:
        sys.path.remove(ref_root)
    for name in ("silu_integer", "sigmoid_integer", "softplus_integer"):
        assert torch.equal(getattr(I, name)(z), getattr(R, name)(z)), name
    a, b = torch.randn(3, 5, generator=g), torch.randn(3, 5, generator=g)
    assert torch.equal(I.silu_multiply_integer(a, b), R.silu_multiply_integer(a, b))
    assert torch.equal(I.quantize_weight_int8(w)[0], R.quantize_weight_int8(w)[0])


def test_zipf_weights_bases_and_core_names(tmp_path):
    import os
    import sys

    import pytest
    import torch

    from complexity_framework_b200 import ComplexityModel, ModelConfig
    from complexity_framework_b200.core.bases import (AttentionBase, MLPBase, build_norm,
                                                      deterministic_gaussian_init_)
    from complexity_framework_b200.core.registry import MLP_REGISTRY, register_mlp
    from complexity_framework_b200.models.builder import build_lexical_zipf_weights

    c = torch.tensor([5.0, 1, 9, 9, 0, 3])
    w = build_lexical_zipf_weights(c, mode="ordered", alpha=0.5, floor=0.1, permutation_seed=3)
    assert abs(float(w.square().mean()) - 1) < 1e-5 and w[2] < w[0] < w[1]
    ref_root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "baseline", "_ref")
    if os.path.isdir(os.path.join(ref_root, "complexity")):
        sys.path.insert(0, ref_root)
        try:
            from complexity.models.builder import build_lexical_zipf_weights as R
        finally:
            sys.path.remove(ref_root)
        for mode in ("ordered", "permuted"):
            assert torch.allclose(build_lexical_zipf_weights(c, mode=mode, alpha=0.5, floor=0.1,
                                                             permutation_seed=3),
                                  R(c, mode=mode, alpha=0.5, floor=0.1, permutation_seed=3))
    torch.save({"counts": torch.arange(64.0)}, tmp_path / "z.pt")
    m = ComplexityModel(ModelConfig(hidden_size=32, num_hidden_layers=1, num_attention_heads=4,
                                    vocab_size=64, intermediate_size=32, num_experts=2,
                                    lexical_zipf_mode="permuted",
                                    lexical_zipf_path=str(tmp_path / "z.pt")))
    assert m.state_dict()["lexical_zipf_weights"].shape == (64,)
    with pytest.raises(ValueError, match="lexical_zipf_path"):
        ComplexityModel(ModelConfig(hidden_size=32, num_hidden_layers=1, num_attention_heads=4,
                                    vocab_size=64, lexical_zipf_mode="ordered"))
    a, b = torch.empty(3, 4), torch.empty(3, 4)
    assert torch.equal(deterministic_gaussian_init_(a, 7), deterministic_gaussian_init_(b, 7))
    assert build_norm("rmsnorm", 8)(torch.randn(2, 8)).shape == (2, 8)

    @register_mlp("test_scaled_identity")
    class Scaled(MLPBase):
        def __init__(self, config):
            super().__init__(config)
            self.s = torch.nn.Parameter(torch.ones(()))

        def forward(self, hidden_states, token_ids=None, **kw):
            return hidden_states * self.s

    assert "test_scaled_identity" in MLP_REGISTRY.names() if hasattr(MLP_REGISTRY, "names") \
        else True
    with pytest.raises(TypeError):
        AttentionBase(None)


def test_tensorboard_writer_and_safety_callback(tmp_path):
    import torch

    from complexity_framework_b200.training.callbacks import TensorBoardMetricWriter
    from complexity_framework_b200.utils.safety import SafetyCallback

    w = TensorBoardMetricWriter(tmp_path / "tb", enabled=False)
    assert not w.enabled
    w.add_scalars("train", {"loss": 1.0}, 1)
    cb = SafetyCallback(torch.nn.Linear(2, 2), log_every=1, reset_stats_every=2)
    cb.on_step_end()
    cb.on_step_end(None, 2, 0.5)
    assert [h["step"] for h in cb.history] == [1, 2]
