"""Sensor-fusion classifier, folds and manifest data path (CPU)."""
import torch

from complexity_framework_b200.generative.sensor_fusion import (
    SensorDataset, SensorRecord, TRHashSensorFusionClassifier, TRHashSensorFusionConfig,
    collate_sensors, load_pretrained_visual_tower, load_sensor_manifest,
    make_cross_subject_folds, resolve_cross_subject_fold, save_sensor_manifest,
    subject_disjoint_records, validate_cross_subject_folds)


def _cfg():
    return TRHashSensorFusionConfig(num_classes=3, hidden_size=64, num_hidden_layers=1,
                                    num_attention_heads=4, num_experts=4, shared_width=128,
                                    expert_width=32, vision_image_size=32, vision_patch_size=8,
                                    vision_hidden_size=32, vision_layers=1, vision_heads=4,
                                    visual_token_grid=2, sequence_tokens=8, classifier_dropout=0.0)


def _inputs(B=3):
    return {"depth": torch.rand(B, 2, 3, 32, 32), "ir": torch.rand(B, 2, 1, 32, 32),
            "imu": torch.randn(B, 20, 45), "skeleton": torch.randn(B, 20, 17, 3)}


def test_fusion_fits_and_handles_missing_streams():
    torch.manual_seed(0)
    m = TRHashSensorFusionClassifier(_cfg())
    x, y = _inputs(), torch.tensor([0, 1, 2])
    opt = torch.optim.AdamW(m.parameters(), 3e-3)
    first = None
    for _ in range(20):
        loss = m(x, y)["loss"]
        opt.zero_grad()
        loss.backward()
        opt.step()
        first = first if first is not None else float(loss)
    assert float(loss) < 0.5 * first
    only_imu = m({"imu": torch.randn(2, 10, 45)})
    assert only_imu["logits"].shape == (2, 3)
    # a visual checkpoint's tower initialises the shared tower
    src = TRHashSensorFusionClassifier(_cfg())
    load_pretrained_visual_tower(m, {"tower." + k: v for k, v in src.vision.state_dict().items()})
    assert torch.equal(m.vision.patch.weight, src.vision.patch.weight)


def test_folds_and_subject_split(tmp_path):
    folds = make_cross_subject_folds(range(1, 11), 5)
    validate_cross_subject_folds(folds)
    assert sorted(s for f in folds for s in f.val_subjects) == list(range(1, 11))
    assert resolve_cross_subject_fold("fold2", folds).val_subjects == (3, 8)
    recs = []
    for i in range(12):
        p = tmp_path / f"imu{i}.pt"
        torch.save(torch.randn(10, 45), p)
        recs.append(SensorRecord({"imu": str(p)}, label=i % 3, subject=i % 6))
    tr, va = subject_disjoint_records(recs, 0.34, seed=1)
    assert not ({r.subject for r in tr} & {r.subject for r in va}) and va
    save_sensor_manifest(recs, str(tmp_path / "m.json"))
    back = load_sensor_manifest(str(tmp_path / "m.json"))
    x, y = collate_sensors([SensorDataset(back)[i] for i in range(3)])
    assert x["imu"].shape == (3, 10, 45) and y.tolist() == [0, 1, 2]
