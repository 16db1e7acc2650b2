"""Device policy and GPU-helper package (CPU behaviour)."""
import pytest
import torch

from complexity_framework_b200 import gpu
from complexity_framework_b200.utils import device as D


def test_device_policy_on_cpu():
    assert D.get_backend("cpu") == "cpu"
    assert D.select_device("auto").type in ("cpu", "cuda")
    for b in ("rocm", "mps"):
        with pytest.raises(RuntimeError):
            D.get_backend(b)
    assert not D.is_mps_available() and not D.is_rocm_available()
    meta = D.backend_metadata("cpu")
    assert meta["name"] == "cpu" and meta["custom_kernels"] is False
    assert D.autocast_dtype(torch.device("cpu")) is None
    with D.autocast(torch.device("cpu")):
        pass
    D.seed_all(3)
    a = torch.rand(2)
    D.seed_all(3)
    assert torch.equal(a, torch.rand(2))
    assert D.custom_kernels_enabled(False) is False


def test_gpu_helpers():
    torch.manual_seed(0)
    x, r = torch.randn(2, 4, 16), torch.randn(2, 4, 16)
    w = torch.rand(16) + 0.5
    y, s = gpu.fused_residual_rmsnorm(x, r, w)
    ref = (x + r) * torch.rsqrt((x + r).pow(2).mean(-1, keepdim=True) + 1e-6) * w
    assert torch.allclose(y, ref, atol=1e-5) and torch.equal(s, x + r)
    g, u = torch.randn(3, 8), torch.randn(3, 8)
    assert torch.allclose(gpu.fused_swiglu(g, u), torch.nn.functional.silu(g) * u)
    n = gpu.FusedRMSNorm(16)
    assert n(x).shape == x.shape
    assert torch.allclose(gpu.upcast_softmax(torch.randn(2, 5)).sum(-1), torch.ones(2))
    m = torch.nn.Linear(1000, 1000)
    m.config = type("C", (), {"hidden_size": 1024, "num_hidden_layers": 16})()
    b = gpu.estimate_max_batch_size(m, seq_len=2048, total_memory_bytes=180 * 2 ** 30)
    assert b >= 1 and (b & (b - 1)) == 0
    assert gpu.apply_gpu_patches(expandable_segments=False)["triton_heuristics"] is False
    with pytest.raises(RuntimeError, match="RCCL"):
        gpu.configure_rccl()
    with gpu.BF16Autocast():
        pass
