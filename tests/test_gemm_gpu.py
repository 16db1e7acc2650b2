"""Numerics of the tcgen05 GEMM against a plain fp32 PyTorch reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu

EPI_STORE, EPI_RESID, EPI_SWIGLU_FWD, EPI_SWIGLU_BWD, EPI_F32, EPI_F32_ACC, EPI_CE_STATS = range(7)


def _C():
    from complexity_framework_b200.ops import require

    return require()


def _operands(M, N, K, a_mn, b_mn, dev="cuda"):
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, generator=g).to(dev, torch.bfloat16)
    b = torch.randn(N, K, generator=g).to(dev, torch.bfloat16)
    A = a.t().contiguous() if a_mn else a
    B = b.t().contiguous() if b_mn else b
    ref = a.float() @ b.float().t()
    return A, B, ref


def _check(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"max rel err {err / scale:.3e}"


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K,bn", [(128, 128, 64, 128), (256, 512, 192, 256),
                                      (296, 384, 200, 128), (1024, 1152, 896, 0)])
def test_gemm_store(M, N, K, bn, a_mn, b_mn):
    C = _C()
    A, B, ref = _operands(M, N, K, a_mn, b_mn)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, a_mn, B, b_mn, M, N, K, EPI_STORE, out=out, bn=bn)
    torch.cuda.synchronize()
    _check(out, ref)


def test_gemm_residual_and_f32():
    C = _C()
    M, N, K = 512, 896, 896
    A, B, ref = _operands(M, N, K, False, False)
    r = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, False, B, False, M, N, K, EPI_RESID, out=out, residual=r, alpha=0.5)
    _check(out, 0.5 * ref + r.float())
    o32 = torch.zeros(M, N, device="cuda")
    C.gemm(A, False, B, False, M, N, K, EPI_F32, out=o32)
    _check(o32, ref, 1e-3)
    C.gemm(A, False, B, False, M, N, K, EPI_F32_ACC, out=o32)
    _check(o32, 2 * ref, 1e-3)


def test_gemm_swiglu_fwd_bwd():
    C = _C()
    M, H, shared, E, W = 512, 256, 256, 4, 64
    act_w = shared + E * W  # 512 -> 4 blocks of 128
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(M, H, generator=g) * 0.5).cuda().bfloat16()
    wg = (torch.randn(act_w, H, generator=g) * 0.05).cuda().bfloat16()
    wu = (torch.randn(act_w, H, generator=g) * 0.05).cuda().bfloat16()
    nb = act_w // 128
    packed = torch.stack([wg.view(nb, 128, H), wu.view(nb, 128, H)], 1).reshape(2 * act_w, H)
    scales = torch.rand(M, E, generator=g).cuda()
    gu = torch.empty(M, 2 * act_w, device="cuda", dtype=torch.bfloat16)
    act = torch.empty(M, act_w, device="cuda", dtype=torch.bfloat16)
    C.gemm(x, False, packed, False, M, 2 * act_w, H, EPI_SWIGLU_FWD, gu=gu, act=act,
           row_scale=scales, shared_width=shared, expert_width=W, n_experts=E, shared_scale=0.7)
    gr = x.float() @ wg.float().t()
    ur = x.float() @ wu.float().t()
    col_scale = torch.cat([torch.full((M, shared), 0.7, device="cuda"),
                           scales.repeat_interleave(W, dim=1)], 1)
    act_ref = torch.nn.functional.silu(gr) * ur * col_scale
    _check(act, act_ref)
    gu_v = gu.view(M, nb, 2, 128)
    _check(gu_v[:, :, 0].reshape(M, act_w), gr)
    _check(gu_v[:, :, 1].reshape(M, act_w), ur)

    # backward: d(act) = dy @ Wd  (Wd: [Hout, act_w] row-major -> B MN-major)
    Hout = 256
    dy = torch.randn(M, Hout, generator=g).cuda().bfloat16()
    wd = (torch.randn(Hout, act_w, generator=g) * 0.05).cuda().bfloat16()
    dgu = torch.empty(M, 2 * act_w, device="cuda", dtype=torch.bfloat16)
    C.gemm(dy, False, wd, True, M, act_w, Hout, EPI_SWIGLU_BWD, out=dgu, gu=gu,
           row_scale=scales, shared_width=shared, expert_width=W, n_experts=E, shared_scale=0.7)
    da = (dy.float() @ wd.float()) * col_scale
    gb = gu_v[:, :, 0].reshape(M, act_w).float()
    ub = gu_v[:, :, 1].reshape(M, act_w).float()
    sg = torch.sigmoid(gb)
    dg_ref = da * ub * sg * (1 + gb * (1 - sg))
    du_ref = da * gb * sg
    dgu_v = dgu.view(M, nb, 2, 128)
    _check(dgu_v[:, :, 0].reshape(M, act_w), dg_ref)
    _check(dgu_v[:, :, 1].reshape(M, act_w), du_ref)


def test_gemm_ce_stats():
    C = _C()
    M, N, K = 256, 1024, 128
    A, B, ref = _operands(M, N, K, False, False)
    bn = 256
    nt = N // 128
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    stats = torch.empty(M, nt, 2, device="cuda")
    C.gemm(A, False, B, False, M, N, K, EPI_CE_STATS, out=out, stats=stats, bn=bn)
    torch.cuda.synchronize()
    _check(out, ref)
    lse = torch.logsumexp(out.float(), dim=1)
    m = stats[..., 0].max(1).values
    s = (stats[..., 1] * torch.exp(stats[..., 0] - m[:, None])).sum(1)
    assert torch.allclose(m + torch.log(s), lse, atol=1e-3, rtol=1e-4)


def test_gemm_no_device_errors():
    from complexity_framework_b200.ops import check_errors

    torch.cuda.synchronize()
    check_errors(0)


@pytest.mark.parametrize("M,N,K", [(896, 3328, 8192), (256, 512, 4096), (6656, 896, 16384)])
def test_gemm_split_k_atomic(M, N, K):
    C = _C()
    A, B, ref = _operands(M, N, K, True, True)
    out = torch.zeros(M, N, device="cuda", dtype=torch.float32)
    C.gemm(A, True, B, True, M, N, K, 7, out=out)
    torch.cuda.synchronize()
    _check(out, ref, 1e-3)


@pytest.mark.parametrize("As,E,W", [(384, 4, 64), (0, 4, 64), (256, 2, 128)])
def test_copy_jobs_pack_unpack(As, E, W):
    """One-launch packing of the TR-Hash MLP weights equals the torch packing,
    and the unpack jobs invert it (fp32 gradients cast to bf16)."""
    from complexity_framework_b200.ops import fused

    torch.manual_seed(0)
    H = 192
    dev = "cuda"
    rnd = lambda *s: torch.randn(*s, device=dev).bfloat16()  # noqa: E731
    sg, su, sd = (rnd(As, H), rnd(As, H), rnd(H, As)) if As else (None, None, None)
    eg, eu, ed = rnd(E, H, W), rnd(E, H, W), rnd(E, W, H)
    gu, down = fused.pack_trhash_weights(sg, su, eg, eu, sd, ed)
    assert torch.equal(gu, fused.pack_gate_up(sg, su, eg, eu))
    assert torch.equal(down, fused.pack_down(sd, ed))
    d_gu = torch.randn(gu.shape, device=dev)
    d_down = torch.randn(down.shape, device=dev)
    got = fused._unpack_trhash_grads((As, E, H, W), d_gu, d_down)
    got_t = fused._unpack_trhash_grads((As, E, H, W), d_gu, d_down.t().contiguous(),
                                       down_transposed=True)
    for a, b in zip(got, got_t):
        assert (a is None and b is None) or torch.equal(a, b)
    ref_in = [t.float().requires_grad_() if t is not None else None
              for t in (sg, su, eg, eu, sd, ed)]
    rg, rd = fused.pack_gate_up(*ref_in[:4]), fused.pack_down(ref_in[4], ref_in[5])
    torch.autograd.backward([rg, rd], [d_gu, d_down])
    for g, r in zip(got, ref_in):
        if r is None:
            assert g is None
        else:
            assert torch.equal(g, r.grad.bfloat16())


def test_trhash_mlp_params_matches_packed():
    from complexity_framework_b200.ops import fused

    torch.manual_seed(1)
    T, H, As, E, W = 512, 256, 256, 4, 64
    dev = "cuda"
    mk = lambda *s: (0.05 * torch.randn(*s, device=dev)).bfloat16().requires_grad_()  # noqa: E731
    params = [mk(As, H), mk(As, H), mk(E, H, W), mk(E, H, W), mk(H, As), mk(E, W, H)]
    x = torch.randn(T, H, device=dev).bfloat16().requires_grad_()
    scales = torch.rand(T, E, device=dev)
    y1 = fused.trhash_mlp_params(x, *params, scales, None, As, W, E, 1.0)
    g = torch.randn_like(y1)
    grads1 = torch.autograd.grad(y1, [x, *params], g)
    gu = fused.pack_gate_up(*params[:4])
    dn = fused.pack_down(params[4], params[5])
    y2 = fused.trhash_mlp(x, gu, dn, scales, None, As, W, E, 1.0)
    grads2 = torch.autograd.grad(y2, [x, *params], g)
    assert torch.equal(y1, y2)
    for a, b in zip(grads1, grads2):
        # same GEMMs; the packed path rounds the weight gradient to bf16 before
        # the autograd scatter, this one after the fp32 split-K sum
        assert float((a.float() - b.float()).abs().max()) <= 1e-2 * float(b.abs().max()) + 1e-6


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (5, 6144, 4096), (64, 4096, 15104),
                                   (100, 896, 3328), (128, 4096, 4096)])
@pytest.mark.parametrize("resid", [False, True])
def test_skinny_gemm_nt(M, N, K, resid):
    """Decode-shaped x @ W^T: swapped operands, split-K fp32 atomics, fused
    transpose/residual/cast pass."""
    from complexity_framework_b200.ops import fused

    assert fused._skinny(M, N, K)
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).cuda().bfloat16()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).cuda().bfloat16()
    r = torch.randn(M, N, generator=g).cuda().bfloat16() if resid else None
    out = fused.gemm_nt(x, w, r, alpha=0.5)
    ref = 0.5 * (x.float() @ w.float().t()) + (r.float() if resid else 0)
    _check(out, ref)
