"""sm_100a flash attention against fp32 PyTorch attention."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(q, k, v, causal, scale):
    B, Hq, S, D = q.shape
    rep = Hq // k.shape[1]
    kf = k.float().repeat_interleave(rep, 1)
    vf = v.float().repeat_interleave(rep, 1)
    s = (q.float() @ kf.transpose(-1, -2)) * scale
    if causal:
        s = s.masked_fill(torch.ones(S, S, device=q.device, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ vf
    return o.transpose(1, 2).reshape(B, S, Hq * D), lse


@pytest.mark.parametrize("B,Hq,Hkv,S,D,causal", [(2, 4, 2, 256, 64, True), (1, 14, 2, 2048, 64, True),
                                                 (2, 4, 4, 384, 128, True), (1, 2, 1, 200, 64, True),
                                                 (2, 4, 2, 256, 64, False)])
def test_flash_forward(B, Hq, Hkv, S, D, causal):
    from complexity_framework_b200.ops.flash import flash_forward

    g = torch.Generator(device="cpu").manual_seed(S + D)
    q = torch.randn(B, Hq, S, D, generator=g).cuda().bfloat16()
    k = torch.randn(B, Hkv, S, D, generator=g).cuda().bfloat16()
    v = torch.randn(B, Hkv, S, D, generator=g).cuda().bfloat16()
    scale = 1 / math.sqrt(D)
    out, lse = flash_forward(q, k, v, causal, scale)
    ro, rl = _ref(q, k, v, causal, scale)
    err = (out.float() - ro).abs().max().item()
    assert err < 2e-2 * ro.abs().max().item() + 1e-2, err
    assert torch.allclose(lse, rl, atol=1e-2, rtol=1e-3)


def test_flash_no_errors():
    from complexity_framework_b200.ops import check_errors

    torch.cuda.synchronize()
    check_errors(0)
