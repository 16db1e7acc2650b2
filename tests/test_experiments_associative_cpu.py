"""Fast-weight memory experiments: parity with the reference's research modules
on identical weights (outputs and carried state over two calls that cross
chunk boundaries), plus the chunked scan against a step-by-step recurrence."""
import os
import sys

import pytest
import torch

from complexity_framework_b200 import experiments as ours

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        from complexity.experiments import shared_associative_attention as m
    except Exception as exc:  # pragma: no cover
        pytest.skip(f"reference import failed: {exc}")
    finally:
        sys.path.remove(REF)
    return m


H, R, V = 32, 16, 97
CASES = [
    ("SharedAssociativeAttention", dict(hidden_size=H, rank=R, vocab_size=V), 300),
    ("SharedAssociativeAttention", dict(hidden_size=H, rank=R, contextual_mix_init=0.3), 300),
    ("SharedContextFusion", dict(hidden_size=H, rank=R, fusion_size=24, vocab_size=V), 300),
    ("StableDeltaAssociativeAttention", dict(hidden_size=H, rank=R, delta_chunk_size=8), 20),
    ("MultiTimescaleDeltaAttention", dict(hidden_size=H, state_rank=R, num_timescales=4,
                                          delta_chunk_size=8), 20),
    ("CollisionNormalizedDeltaAttention", dict(hidden_size=H, state_rank=R, vocab_size=V,
                                               delta_chunk_size=8), 20),
    ("LexicalValueDeltaAttention", dict(hidden_size=H, state_rank=R, delta_chunk_size=8), 20),
    ("LexicalForgeDeltaAttention", dict(hidden_size=H, state_rank=R, delta_chunk_size=8), 20),
    ("CollisionNormalizedLexicalForgeDeltaAttention", dict(hidden_size=H, state_rank=R,
                                                           delta_chunk_size=8), 20),
    ("PositionAwareCollisionForgeDeltaAttention", dict(hidden_size=H, state_rank=R,
                                                       delta_chunk_size=8), 20),
    ("MultiOrderLexicalDeltaAttention", dict(hidden_size=H, head_rank=R, orders=(1, 2, 3),
                                             delta_chunk_size=8), 20),
]


def _perturb(m):
    """Move the gates and scales off their initial values so every term matters."""
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.ndim <= 1:
                p.add_(0.3 * torch.randn(p.shape, generator=g))


@pytest.mark.parametrize("name,kw,L", CASES, ids=[f"{c[0]}{i}" for i, c in enumerate(CASES)])
def test_matches_reference(ref, name, kw, L):
    torch.manual_seed(0)
    rm = getattr(ref, name)(**kw)
    _perturb(rm)
    mm = getattr(ours, name)(**kw)
    missing = mm.load_state_dict(rm.state_dict(), strict=True)
    assert not missing.missing_keys and not missing.unexpected_keys
    forge = "Forge" in name
    if forge:
        emb = torch.nn.Embedding(V, 16)
        rm.attach_token_scale(emb)
        mm.attach_token_scale(emb)
    g = torch.Generator().manual_seed(1)
    B = 2
    sr = rm.initial_state(B, device=torch.device("cpu"), dtype=torch.float32)
    sm = mm.initial_state(B, device=torch.device("cpu"), dtype=torch.float32)
    for _ in range(2):
        h = torch.randn(B, L, H, generator=g)
        ids = torch.randint(0, V, (B, L), generator=g)
        orr, sr = rm(h, ids, sr)
        om, sm = mm(h, ids, sm)
        assert torch.allclose(om, orr, atol=2e-5, rtol=1e-4), (om - orr).abs().max()
        assert len(sr) == len(sm)
        for a, b in zip(sm, sr):
            if a.is_floating_point():
                assert torch.allclose(a, b.float(), atol=2e-5, rtol=1e-4), (a - b).abs().max()
            else:
                assert torch.equal(a, b)


@pytest.mark.parametrize("delta", [False, True])
def test_chunk_scan_matches_recurrence(delta):
    g = torch.Generator().manual_seed(3)
    B, C, r, n = 3, 11, 6, 5
    q, k = torch.randn(B, C, r, generator=g), torch.randn(B, C, r, generator=g) * 0.3
    v, S0 = torch.randn(B, C, n, generator=g), torch.randn(B, r, n, generator=g)
    d, w = torch.tensor([0.9, 0.97, 0.5]), torch.tensor([0.4, 0.8, 0.6])
    reads, S = ours.chunk_scan(q, k, v, S0, d, w, delta)
    St, want = S0.clone(), []
    for t in range(C):
        want.append(torch.einsum("br,brn->bn", q[:, t], St))
        e = v[:, t] - (torch.einsum("br,brn->bn", k[:, t], St) if delta else 0)
        St = d[:, None, None] * St + w[:, None, None] * k[:, t, :, None] * e[:, None, :]
    assert torch.allclose(reads, torch.stack(want, 1), atol=1e-5)
    assert torch.allclose(S, St, atol=1e-5)


def test_gradients_flow():
    m = ours.PositionAwareCollisionForgeDeltaAttention(H, 16, delta_chunk_size=8)
    h = torch.randn(2, 12, H, requires_grad=True)
    out, _ = m(h, torch.randint(0, V, (2, 12)), m.initial_state(2))
    out.square().sum().backward()
    assert h.grad is not None and torch.isfinite(h.grad).all()
    assert all(p.grad is not None for n, p in m.named_parameters()
               if not n.startswith("forge_")), [n for n, p in m.named_parameters() if p.grad is None]
