"""Grouped tcgen05 routed experts (wide experts) against fp32 reference math.

Forward output, input gradient and gate/up/down weight gradients of
``GroupedExpertsFn`` are compared with ``reference_topk_swiglu`` evaluated in
fp32 on the same bf16 inputs, at a small shape and at the expert shapes of
the 1B (16 experts of width 256, hidden 2048) and 7B (8 experts of width 512,
hidden 4096) configurations.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(a, b, what, rel=2e-2):
    err = (a.float() - b.float()).abs().max().item()
    tol = rel * b.float().abs().max().item() + 1e-3
    assert err < tol, f"{what}: max err {err:.4g} > {tol:.4g}"


@pytest.mark.parametrize("T,H,E,W,strategy", [(1000, 256, 4, 128, "zipf"),
                                              (4096, 2048, 16, 256, "zipf"),
                                              (2048, 4096, 8, 512, "uniform")])
def test_grouped_experts_match_reference(T, H, E, W, strategy):
    from complexity_framework_b200.ops import check_errors
    from complexity_framework_b200.ops.grouped import GroupedExpertsFn
    from complexity_framework_b200.tr_hash.engine import reference_topk_swiglu

    g = torch.Generator().manual_seed(T + E)
    k = 2
    if strategy == "zipf":  # skewed expert loads, some experts nearly empty
        p = torch.arange(1, E + 1, dtype=torch.float64).pow(-1.1)
        r0 = torch.multinomial(p / p.sum(), T, replacement=True, generator=g)
    else:
        r0 = torch.randint(0, E, (T,), generator=g)
    r1 = (r0 + 1 + torch.randint(0, E - 1, (T,), generator=g)) % E
    routes = torch.stack([r0, r1]).cuda()
    slot_w = torch.tensor([0.6, 0.4]).cuda()
    x = (torch.randn(T, H, generator=g) * 0.5).cuda().bfloat16()
    gate = (torch.randn(E, H, W, generator=g) * H ** -0.5).cuda().bfloat16()
    up = (torch.randn(E, H, W, generator=g) * H ** -0.5).cuda().bfloat16()
    down = (torch.randn(E, W, H, generator=g) * W ** -0.5).cuda().bfloat16()
    dout = torch.randn(T, H, generator=g).cuda().bfloat16()

    leaves = [t.clone().requires_grad_() for t in (x, gate, up, down)]
    out = GroupedExpertsFn.apply(leaves[0], routes, slot_w, *leaves[1:])
    out.backward(dout)
    torch.cuda.synchronize()
    check_errors(0)

    ref_leaves = [t.float().requires_grad_() for t in (x, gate, up, down)]
    ref = reference_topk_swiglu(ref_leaves[0], routes, *ref_leaves[1:],
                                slot_w[:, None].expand_as(routes))
    ref.backward(dout.float())
    _close(out, ref, "out")
    for name, a, b in zip(("dx", "dgate", "dup", "ddown"), leaves, ref_leaves):
        _close(a.grad, b.grad, name)


def test_plan_is_stable_and_padded():
    import complexity_framework_b200._C as C

    T, E = 3000, 8
    g = torch.Generator().manual_seed(0)
    routes = torch.stack([torch.randint(0, E, (T,), generator=g),
                          torch.randint(0, E, (T,), generator=g)]).cuda()
    slot_w = torch.tensor([0.7, 0.3]).cuda()
    seg, tiles, row_token, row_weight, token_pos = C.moe_plan(routes, E, slot_w)
    seg, tiles, row_token, row_weight, token_pos = (t.cpu() for t in
                                                    (seg, tiles, row_token, row_weight, token_pos))
    flat = routes.cpu().reshape(-1)
    counts = torch.bincount(flat, minlength=E)
    assert torch.all(seg[1:] - seg[:-1] == (counts + 255) // 256 * 256)
    for e in range(E):
        rows = torch.arange(int(seg[e]), int(seg[e]) + int(counts[e]))
        want = torch.nonzero(flat == e).flatten()          # assignment order kept
        assert torch.equal(token_pos[want].long(), rows)
        assert torch.equal(row_token[rows].long(), want % T)
        assert torch.allclose(row_weight[rows], slot_w.cpu()[want // T])
        assert torch.all(row_token[int(seg[e]) + int(counts[e]):int(seg[e + 1])] == -1)
        assert torch.all(tiles[int(seg[e]) // 256:int(seg[e + 1]) // 256] == e)
    assert torch.all(tiles[int(seg[E]) // 256:] == -1)
