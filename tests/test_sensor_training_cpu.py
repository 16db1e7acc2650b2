"""Sensor-fusion training: per-sample modality masks, augmentation and
imbalance helpers, objectives (parity with the reference's functions where
their inputs coincide), and a short training run."""
import math
import os
import sys

import pytest
import torch

from complexity_framework_b200.generative import sensor_training as T
from complexity_framework_b200.generative.sensor_fusion import (SENSOR_MODALITIES, SensorRecord,
                                                                TRHashSensorFusionClassifier,
                                                                TRHashSensorFusionConfig,
                                                                collate_sensors_masked)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _cfg(**kw):
    base = dict(num_classes=3, hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
                num_experts=4, shared_width=128, expert_width=32, vision_image_size=32,
                vision_patch_size=8, vision_hidden_size=32, vision_layers=1, vision_heads=4,
                visual_token_grid=2, sequence_tokens=8, classifier_dropout=0.0)
    base.update(kw)
    return TRHashSensorFusionConfig(**base)


def _sample(label, streams, g):
    x = {}
    if "depth" in streams:
        x["depth"] = torch.rand(2, 3, 32, 32, generator=g) * 0.2 + 0.3 * label
    if "imu" in streams:
        x["imu"] = torch.randn(12, 45, generator=g) * 0.1 + label
    if "skeleton" in streams:
        x["skeleton"] = torch.randn(12, 17, 3, generator=g) * 0.1 - label
    return x, label


def test_masked_forward_ignores_absent_streams():
    torch.manual_seed(0)
    m = TRHashSensorFusionClassifier(_cfg(modality_gate=True)).eval().requires_grad_(False)
    g = torch.Generator().manual_seed(1)
    samples = [_sample(0, ("depth", "imu"), g), _sample(1, ("imu",), g)]
    inputs, masks, labels = collate_sensors_masked(samples)
    assert masks["depth"].tolist() == [True, False]
    out = m(inputs, masks=masks)
    assert out["modality_mask"][1, SENSOR_MODALITIES.index("depth")] == False  # noqa: E712
    assert float(out["modality_weights"][1].sum()) == pytest.approx(1.0)
    # the absent stream's content cannot change the second sample's prediction
    inputs2 = dict(inputs)
    inputs2["depth"] = inputs["depth"].clone()
    inputs2["depth"][1] = torch.rand_like(inputs2["depth"][1])
    out2 = m(inputs2, masks=masks)
    assert torch.allclose(out["logits"][1], out2["logits"][1], atol=1e-5)
    alone = m({"imu": inputs["imu"][1:]})
    assert torch.allclose(out["logits"][1], alone["logits"][0], atol=1e-5)
    with pytest.raises(ValueError, match="at least one"):
        m(inputs, masks={"depth": torch.tensor([True, False]), "imu": torch.tensor([True, False])})


def test_helpers():
    assert [T.augmentation_scale(e, total_epochs=10, clean_finetune_epochs=4)
            for e in (5, 6, 7, 9)] == [1.0, 1.0, 0.75, 0.25]
    masks = {"a": torch.tensor([True, True, False]), "b": torch.tensor([False, True, True])}
    torch.manual_seed(0)
    d = T.apply_modality_dropout(masks, 0.9)
    keep = torch.stack([d["a"], d["b"]], 1)
    have = torch.stack([masks["a"], masks["b"]], 1)
    assert bool(keep.any(1).all()) and bool((~keep | have).all())
    w = T.normalize_bounded_weights(torch.tensor([1.0, 1, 1, 10]), minimum=0.5, maximum=2.0)
    assert float(w.mean()) == pytest.approx(1.0, abs=1e-6) and float(w.max()) <= 2.0
    recs = [SensorRecord({"imu": ""}, l, s) for l, s in [(0, 1), (0, 1), (0, 2), (1, 1)]]
    cw, counts = T.build_class_weights(recs, num_classes=3, mode="inverse", device="cpu")
    assert counts.tolist() == [3, 1, 0] and cw[2] == 0 and float(cw[:2].mean()) == pytest.approx(1)
    sw = T.build_sample_loss_weights(recs, num_classes=3, mode="inverse-2d")
    assert float(sw.mean()) == pytest.approx(1.0) and sw[3] > sw[0]
    conf = torch.tensor([[3, 1], [0, 4]])
    r = T.classification_metrics_from_confusion(conf)
    assert r["accuracy"] == pytest.approx(7 / 8)


def test_objectives_match_reference():
    if not os.path.isdir(os.path.join(REF, "complexity")):
        pytest.skip("reference install not present")
    sys.path.insert(0, REF)
    try:
        from complexity.generative.sensor_fusion import training as R
    except Exception as exc:  # pragma: no cover
        pytest.skip(f"reference import failed: {exc}")
    finally:
        sys.path.remove(REF)
    g = torch.Generator().manual_seed(2)
    B, M, C = 6, len(SENSOR_MODALITIES), 5
    logits = torch.randn(B, M, C, generator=g)
    mask = {n: torch.rand(B, generator=g) > 0.3 for n in SENSOR_MODALITIES}
    mask[SENSOR_MODALITIES[0]] = torch.ones(B, dtype=torch.bool)
    labels = torch.randint(0, C, (B,), generator=g)
    sw = torch.rand(B, generator=g) + 0.5
    a = T.auxiliary_modality_loss(logits, mask, labels, sw, class_weights=None,
                                  label_smoothing=0.1)
    b = R.auxiliary_modality_loss(logits, mask, labels, sw, class_weights=None,
                                  label_smoothing=0.1)
    assert torch.allclose(a, b, atol=1e-6)
    gw = torch.rand(B, M, generator=g).softmax(1)
    a = T.modality_gate_calibration_loss(logits, gw, mask, labels, sw, quality_temperature=0.7,
                                         target_smoothing=0.1, label_smoothing=0.0)
    b = R.modality_gate_calibration_loss(logits, gw, mask, labels, sw, quality_temperature=0.7,
                                         target_smoothing=0.1, label_smoothing=0.0)
    assert torch.allclose(a, b, atol=1e-6)
    feats = torch.randn(8, 16, generator=g)
    lab = torch.tensor([0, 0, 1, 1, 2, 3, 3, 3])
    assert torch.allclose(T.supervised_contrastive_loss(feats, lab, temperature=0.2),
                          R.supervised_contrastive_loss(feats, lab, temperature=0.2), atol=1e-6)
    wl = torch.randn(B, C, generator=g)
    assert torch.allclose(T.weighted_cross_entropy(wl, labels, sw, label_smoothing=0.05),
                          R.weighted_cross_entropy(wl, labels, sw, class_weights=None,
                                                   label_smoothing=0.05), atol=1e-6)
    w = torch.tensor([0.2, 1.0, 3.0, 7.0], dtype=torch.float64)
    assert torch.allclose(T.normalize_bounded_weights(w, minimum=0.3, maximum=2.5),
                          R._normalize_bounded_weights(w, minimum=0.3, maximum=2.5))


def test_training_run_learns(tmp_path):
    g = torch.Generator().manual_seed(0)
    combos = [("depth", "imu", "skeleton"), ("imu",), ("depth", "skeleton")]
    data, recs = [], []
    for i in range(36):
        lab, subj = i % 3, i % 4
        data.append((_sample(lab, combos[i % 3], g), subj))
        recs.append(SensorRecord({k: "" for k in combos[i % 3]}, lab, subj))

    def batches(items):
        out = []
        for j in range(0, len(items), 6):
            chunk = items[j:j + 6]
            inputs, masks, labels = collate_sensors_masked([c[0] for c in chunk])
            out.append((inputs, masks, labels, torch.tensor([c[1] for c in chunk])))
        return out

    torch.manual_seed(0)
    m = TRHashSensorFusionClassifier(_cfg(modality_gate=True))
    cfg = T.SensorTrainConfig(epochs=4, learning_rate=3e-3, warmup_steps=2,
                              sample_weighting="inverse-sqrt-2d", gate_calibration_weight=0.1,
                              contrastive_weight=0.1, clean_finetune_epochs=2,
                              output=str(tmp_path))
    s = T.train_sensor_fusion(m, batches(data), batches(data[:18]), recs, cfg)
    h = s["history"]
    assert all(math.isfinite(e["train_loss"]) for e in h) and h[-1]["aug_scale"] == 0.5
    assert s["best_macro_f1"] > 0.5 and (tmp_path / "best_model.pt").exists()
