"""muP coordinate check: with the muP knobs on, per-coordinate RMS of the
residual stream and of the embeddings stays flat as the width grows; the
standard parametrisation drifts; the output multiplier shrinks wide logits.

Same claims as complexity/tests/test_mup_coordinate_check.py (widths 256 /
512 / 1024 against base width 256, one fp32 forward + backward).
"""
import pytest
import torch
import torch.nn.functional as F

from complexity_framework_b200 import ComplexityModel, ModelConfig

WIDTHS = (256, 512, 1024)
FLAT = 0.30      # largest relative spread accepted under muP
DRIFT = 0.40     # smallest spread expected without it


def _rms(t: torch.Tensor) -> float:
    return float(t.detach().norm() / t.numel() ** 0.5)


def _spread(v):
    return (max(v) - min(v)) / (sum(v) / len(v))


_CACHE = {}


def _probe(width: int, mup: bool):
    key = (width, mup)
    if key in _CACHE:
        return _CACHE[key]
    cfg = ModelConfig(hidden_size=width, num_hidden_layers=4, num_attention_heads=8,
                      num_key_value_heads=4, intermediate_size=int(width * 8 / 3 / 64) * 64,
                      vocab_size=2048, max_position_embeddings=128, attention_type="gqa",
                      mlp_type="dense_deterministic", norm_type="rmsnorm", use_qk_norm=True,
                      use_mup_init=mup, use_mup_attn_scale=mup, use_mup_output_mult=mup,
                      mup_base_width=256)
    torch.manual_seed(0)
    model = ComplexityModel(cfg).float().eval()
    torch.manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (2, 32))
    out = model(ids, return_hidden_states=True)
    logits = out["logits"]
    F.cross_entropy(logits.reshape(-1, cfg.vocab_size), torch.zeros(64, dtype=torch.long)).backward()
    hs = [_rms(h) for h in out["hidden_states"]]
    r = {"embed": hs[0], "mid": hs[len(hs) // 2], "logits": _rms(logits),
         "embed_grad": _rms(model.embed_tokens.weight.grad)}
    _CACHE[key] = r
    return r


def test_mup_residual_stream_is_width_invariant():
    assert _spread([_probe(w, True)["mid"] for w in WIDTHS]) < FLAT


def test_mup_embedding_rms_is_width_invariant():
    assert _spread([_probe(w, True)["embed"] for w in WIDTHS]) < FLAT


def test_standard_parametrisation_drifts():
    mid = [_probe(w, False)["mid"] for w in WIDTHS]
    grad = [_probe(w, False)["embed_grad"] for w in WIDTHS]
    assert max(_spread(mid), _spread(grad)) > DRIFT


def test_output_multiplier_shrinks_wide_logits():
    ratio = _probe(WIDTHS[-1], True)["logits"] / _probe(WIDTHS[0], True)["logits"]
    assert ratio < 1.2 / (WIDTHS[-1] / WIDTHS[0]) ** 0.5
