"""Numerics of the memory-bound sm_100a kernels against fp32 PyTorch references:
RMSNorm fwd/bwd and the fused per-head QK-RMSNorm + RoPE + head-major scatter."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rms_ref(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()


@pytest.mark.parametrize("skip", [False, True])
@pytest.mark.parametrize("T,H", [(4096, 896), (1000, 256), (333, 512), (64, 1024), (77, 200),
                                 (300, 2048)])
def test_rmsnorm_fwd_bwd(T, H, skip):
    from complexity_framework_b200.ops.fused import rmsnorm, rmsnorm_skip

    torch.manual_seed(0)
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_()
    g = torch.randn(T, H, device="cuda").bfloat16()
    gs = torch.randn(T, H, device="cuda").bfloat16()
    if skip:  # second output is the residual stream; its gradient joins in the kernel
        y, xs = rmsnorm_skip(x, w, 1e-6)
        torch.autograd.backward([y, xs], [g, gs])
    else:
        y = rmsnorm(x, w, 1e-6)
        y.backward(g)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = _rms_ref(xr, wr, 1e-6)
    if skip:
        torch.autograd.backward([yr, xr * 1.0], [g.float(), gs.float()])
    else:
        yr.backward(g.float())
    assert (y.float() - yr).abs().max() < 3e-2
    assert (x.grad.float() - xr.grad).abs().max() / xr.grad.abs().max() < 2e-2
    assert (w.grad.float() - wr.grad).abs().max() / wr.grad.abs().max() < 2e-2


def _rope_ref(x, cos, sin, pos):
    # x [B, H, S, D]; cos/sin [maxpos, D/2]
    c = torch.cat([cos, cos], -1)[pos][:, None]  # [B,1,S,D]
    s = torch.cat([sin, sin], -1)[pos][:, None]
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], -1)
    return x * c + rot * s


@pytest.mark.parametrize("D,Hq,Hkv,qk_norm", [(64, 14, 2, True), (128, 8, 8, True),
                                               (64, 4, 1, True), (64, 14, 2, False),
                                               (128, 64, 8, True)])
def test_qk_norm_rope_fwd_bwd(D, Hq, Hkv, qk_norm):
    from complexity_framework_b200.ops.fused import qk_norm_rope

    torch.manual_seed(0)
    B, S = 2, 300
    dev = "cuda"
    kqv = torch.randn(B, S, (Hq + 2 * Hkv) * D, device=dev).bfloat16().requires_grad_()
    qw = (1 + 0.1 * torch.randn(D, device=dev)).bfloat16().requires_grad_()
    kw = (1 + 0.1 * torch.randn(D, device=dev)).bfloat16().requires_grad_()
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=dev).float() / D))
    fr = torch.outer(torch.arange(512, device=dev).float(), inv)
    cos, sin = fr.cos().contiguous(), fr.sin().contiguous()
    pos = torch.arange(S, device=dev, dtype=torch.int32).repeat(B, 1).contiguous()
    q, k, v = qk_norm_rope(kqv, qw, kw, cos, sin, pos, Hq, Hkv, D, 1e-6, qk_norm)
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    (q.float() * gq).sum().add((k.float() * gk).sum()).add((v.float() * gv).sum()).backward()

    kr = kqv.detach().float().requires_grad_()
    qwr = qw.detach().float().requires_grad_()
    kwr = kw.detach().float().requires_grad_()
    kk, qq, vv = kr.split([Hkv * D, Hq * D, Hkv * D], -1)
    qh = qq.view(B, S, Hq, D).transpose(1, 2)
    kh = kk.view(B, S, Hkv, D).transpose(1, 2)
    vh = vv.view(B, S, Hkv, D).transpose(1, 2)
    posl = pos.long()
    nq = _rms_ref(qh, qwr, 1e-6) if qk_norm else qh
    nk = _rms_ref(kh, kwr, 1e-6) if qk_norm else kh
    qr = _rope_ref(nq, cos, sin, posl)
    kr2 = _rope_ref(nk, cos, sin, posl)
    (qr * gq.float()).sum().add((kr2 * gk.float()).sum()).add((vh * gv.float()).sum()).backward()
    for a, b in ((q, qr), (k, kr2), (v, vh)):
        assert (a.float() - b).abs().max() < 5e-2
    rel = lambda a, b: float((a.float() - b).abs().max() / b.abs().max())  # noqa: E731
    assert rel(kqv.grad, kr.grad) < 2e-2
    if qk_norm:
        assert rel(qw.grad, qwr.grad) < 2e-2
        assert rel(kw.grad, kwr.grad) < 2e-2


@pytest.mark.parametrize("T,H,V", [(300, 128, 1056), (1024, 256, 4096)])
def test_linear_cross_entropy_matches_torch(T, H, V):
    """Fused linear CE (GEMM partial stats + loss/grad kernel) against fp32 torch,
    with ignored targets and a vocabulary that is not a multiple of 256."""
    import torch.nn.functional as F

    from complexity_framework_b200.ops.fused import linear_cross_entropy

    torch.manual_seed(0)
    h = torch.randn(T, H, device="cuda").bfloat16().requires_grad_()
    w = (0.05 * torch.randn(V, H, device="cuda")).bfloat16().requires_grad_()
    t = torch.randint(0, V, (T,), device="cuda")
    t[::7] = -100
    loss = linear_cross_entropy(h, w, t)
    (2.0 * loss).backward()
    hr = h.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    lr = F.cross_entropy(hr @ wr.t(), t, ignore_index=-100)
    (2.0 * lr).backward()
    assert abs(float(loss) - float(lr)) < 2e-2
    rel = lambda a, b: float((a.float() - b).abs().max() / b.abs().max())  # noqa: E731
    assert rel(h.grad, hr.grad) < 3e-2
    assert rel(w.grad, wr.grad) < 3e-2


def test_fused_adamw_matches_torch():
    """Flat fp32-master AdamW kernel (8-wide vectors plus ragged tail, device
    clip coefficient) against torch.optim.AdamW on fp32 copies."""
    from complexity_framework_b200.training.optim import FusedAdamW

    torch.manual_seed(0)
    shapes = [(1000, 37), (129,), (64, 64), (7,)]
    ps = [torch.nn.Parameter(torch.randn(s, device="cuda").bfloat16()) for s in shapes]
    ref = [torch.nn.Parameter(p.detach().float().clone()) for p in ps]
    opt = FusedAdamW(ps, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    ropt = torch.optim.AdamW(ref, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, eps=1e-8)
    for step in range(3):
        grads = [torch.randn(s, device="cuda") for s in shapes]
        for p, g in zip(ps, grads):
            p.grad = g.bfloat16()
        opt.clip_grad_norm_(1.0)
        opt.step(clip=True)
        opt.zero_grad()
        gb = [g.bfloat16().float() for g in grads]
        total = torch.sqrt(sum((g * g).sum() for g in gb))
        coef = min(1.0, 1.0 / (float(total) + 1e-6))
        for r, g in zip(ref, gb):
            r.grad = g * coef
        ropt.step()
    for p, r in zip(ps, ref):
        master = opt.state[p]["master"]
        assert float((master.reshape(r.shape) - r.detach()).abs().max()) < 1e-4
        assert float((p.detach().float() - r.detach()).abs().max()) < 2e-2


@pytest.mark.parametrize("H", [256, 896, 2048])
def test_embedding_backward_sorted_and_tied_head(H):
    """Embedding grad (sorted-run accumulation, Zipf-like hot ids) and the tied
    LM-head hand-off (CE weight gradient summed into the embedding backward)
    against torch."""
    import torch.nn.functional as F

    from complexity_framework_b200.ops.fused import embedding, linear_cross_entropy

    torch.manual_seed(0)
    V, T = 1024, 4096
    ids = torch.randint(0, V, (T,), device="cuda")
    ids[::3] = 7  # a hot id
    ids[1::5] = 0
    w = (0.05 * torch.randn(V, H, device="cuda")).bfloat16().requires_grad_()
    tgt = torch.randint(0, V, (T,), device="cuda")
    x = embedding(ids.view(4, -1), w)
    h = (x.float() * 1.5).bfloat16().reshape(T, H)
    loss = linear_cross_entropy(h, w, tgt)
    loss.backward()
    wr = w.detach().float().requires_grad_()
    hr = wr[ids] * 1.5
    lr = F.cross_entropy(hr @ wr.t(), tgt)
    lr.backward()
    err = float((w.grad.float() - wr.grad).abs().max() / wr.grad.abs().max())
    assert err < 3e-2, err
    assert getattr(w, "_cfb_pending_grad", None) is None
