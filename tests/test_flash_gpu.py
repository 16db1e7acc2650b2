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


def _ref_grads(q, k, v, causal, scale, dout):
    """fp32 autograd gradients of attention with K/V repeated per group."""
    qf = q.detach().float().requires_grad_()
    kf = k.detach().float().requires_grad_()
    vf = v.detach().float().requires_grad_()
    o, _ = _ref(qf, kf, vf, causal, scale)
    o.backward(dout.float())
    return o, qf.grad, kf.grad, vf.grad


def _close(a, b, what):
    err = (a.float() - b).abs().max().item()
    tol = 2e-2 * b.abs().max().item() + 2e-3
    assert err < tol, f"{what}: max err {err} > {tol}"


@pytest.mark.parametrize("B,Hq,Hkv,S,D,causal,token_major", [
    (2, 4, 2, 256, 64, True, True), (1, 14, 2, 2048, 64, True, True),
    (2, 4, 4, 384, 128, True, True), (1, 2, 1, 200, 64, True, False),
    (2, 4, 2, 256, 64, False, False), (1, 2, 2, 130, 128, True, False),
    (1, 4, 1, 320, 128, False, True)])
def test_flash_backward(B, Hq, Hkv, S, D, causal, token_major):
    from complexity_framework_b200.ops.flash import flash_attention

    g = torch.Generator(device="cpu").manual_seed(7 * S + D)
    if token_major:  # the layout the QK-norm/RoPE kernel writes
        q = torch.randn(B, S, Hq, D, generator=g).cuda().bfloat16().transpose(1, 2)
    else:
        q = torch.randn(B, Hq, S, D, generator=g).cuda().bfloat16()
    k = torch.randn(B, Hkv, S, D, generator=g).cuda().bfloat16()
    v = torch.randn(B, Hkv, S, D, generator=g).cuda().bfloat16()
    dout = torch.randn(B, S, Hq * D, generator=g).cuda().bfloat16()
    scale = 1 / math.sqrt(D)
    qg, kg, vg = (t.detach().requires_grad_() for t in (q, k, v))
    out = flash_attention(qg, kg, vg, causal=causal, scale=scale)
    out.backward(dout)
    ro, rdq, rdk, rdv = _ref_grads(q, k, v, causal, scale, dout)
    _close(out, ro, "out")
    _close(qg.grad, rdq, "dq")
    _close(kg.grad, rdk, "dk")
    _close(vg.grad, rdv, "dv")
    if token_major:  # dq keeps q's token-major memory layout
        assert qg.grad.transpose(1, 2).is_contiguous()
    from complexity_framework_b200.ops import check_errors

    torch.cuda.synchronize()
    check_errors(0)
