"""Reference-API multimodal towers: shapes, and parity with the reference's
modules on identical weights (state dicts load across unchanged)."""
import os
import sys

import pytest
import torch

from complexity_framework_b200 import multimodal as mm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        import complexity.multimodal as m
    except Exception as exc:  # pragma: no cover
        pytest.skip(f"reference import failed: {exc}")
    finally:
        sys.path.remove(REF)
    return m


g = torch.Generator().manual_seed(0)
IMG = torch.randn(2, 3, 32, 32, generator=g)
MEL = torch.randn(2, 16, 40, generator=g)
VID = torch.randn(2, 3, 4, 32, 32, generator=g)
TXT = torch.randn(2, 5, 64, generator=g)
OTH = torch.randn(2, 7, 64, generator=g)

CASES = [
    ("VisionEncoder", dict(image_size=32, patch_size=8, hidden_size=64, num_layers=2,
                           num_heads=4, num_experts=4, output_dim=48), (IMG,), {}),
    ("VisionEncoder", dict(image_size=32, patch_size=8, hidden_size=64, num_layers=1,
                           num_heads=4, num_experts=1), (IMG,), {"return_all_features": True}),
    ("CLIPVisionEncoder", dict(image_size=32, patch_size=8, hidden_size=64, num_layers=1,
                               num_heads=4, output_dim=32, num_experts=2), (IMG,), {}),
    ("SigLIPEncoder", dict(image_size=32, patch_size=8, hidden_size=64, num_layers=1,
                           num_heads=4, output_dim=32, num_experts=2), (IMG,), {}),
    ("AudioEncoder", dict(n_mels=16, hidden_size=64, num_layers=2, num_heads=4,
                          num_experts=4), (MEL,), {"return_all_features": True}),
    ("AudioEncoder", dict(n_mels=16, hidden_size=64, num_layers=1, num_heads=4,
                          encoder_type="mel", num_experts=2, output_dim=32), (MEL,), {}),
    ("VideoEncoder", dict(image_size=32, patch_size=8, num_frames=4, temporal_patch_size=2,
                          hidden_size=64, num_layers=2, num_heads=4, num_experts=4),
     (VID,), {"return_all_features": True}),
    ("CrossAttentionFusion", dict(hidden_size=64, num_heads=4, num_layers=2, dropout=0.0,
                                  num_experts=4), (TXT, OTH), {}),
    ("PerceiverResampler", dict(hidden_size=64, num_latents=6, num_heads=4, num_layers=1,
                                dropout=0.0, num_experts=1), (OTH,), {}),
    ("GatedFusion", dict(hidden_size=64, num_modalities=2), (TXT, TXT.flip(1)), {}),
    ("ConcatProjection", dict(hidden_size=64, dropout=0.0), (TXT, OTH), {}),
    ("VisionLanguageConnector", dict(vision_hidden_size=64, language_hidden_size=32,
                                     connector_type="resampler"), (OTH,), {}),
]


@pytest.mark.parametrize("name,kw,args,fkw", CASES, ids=[f"{c[0]}{i}" for i, c in enumerate(CASES)])
def test_matches_reference(ref, name, kw, args, fkw):
    torch.manual_seed(1)
    r = getattr(ref, name)(**kw).eval()
    o = getattr(mm, name)(**kw).eval()
    res = o.load_state_dict(r.state_dict(), strict=True)
    assert not res.missing_keys and not res.unexpected_keys
    with torch.no_grad():
        a, b = o(*args, **fkw), r(*args, **fkw)
    assert a.shape == b.shape
    assert torch.allclose(a, b, atol=2e-5, rtol=1e-4), (a - b).abs().max()


@pytest.mark.parametrize("fusion_type", ["cross_attention", "gated", "concat", "perceiver"])
def test_multimodal_fusion_matches_reference(ref, fusion_type):
    kw = dict(hidden_size=64, num_heads=4, num_layers=1, fusion_type=fusion_type,
              num_latents=4, dropout=0.0, num_experts=2)
    torch.manual_seed(2)
    r = ref.MultimodalFusion(**kw).eval()
    o = mm.MultimodalFusion(**kw).eval()
    o.load_state_dict(r.state_dict())
    with torch.no_grad():
        assert torch.allclose(o(TXT, OTH), r(TXT, OTH), atol=2e-5)


def test_siglip_loss_and_clip_scale():
    s = mm.SigLIPEncoder(image_size=32, patch_size=8, hidden_size=64, num_layers=1, num_heads=4,
                         output_dim=64, num_experts=1)
    f = s(IMG)
    assert torch.allclose(f.norm(dim=-1), torch.ones(2), atol=1e-5)
    lo = s.compute_loss(f, f)
    hi = s.compute_loss(f, -f)
    assert lo < hi
    c = mm.CLIPVisionEncoder(image_size=32, patch_size=8, hidden_size=64, num_layers=1,
                             num_heads=4, output_dim=32)
    assert abs(float(c.get_logit_scale()) - 1 / 0.07) < 1e-3


def test_preprocessor_and_frame_limit():
    pre = mm.AudioPreprocessor(n_mels=16, n_fft=64, hop_length=16)
    mel = pre(torch.randn(2, 800))
    assert mel.shape == (2, 16, 51)
    assert abs(float(mel.mean())) < 1e-4
    w = mm.WhisperEncoder(n_mels=16, hidden_size=32, num_layers=1, num_heads=4, max_length=10)
    with pytest.raises(ValueError, match="max_length"):
        w(torch.randn(1, 16, 40))
