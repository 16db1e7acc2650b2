"""Graph-structured skeleton / IMU encoders and gradient reversal in the
sensor-fusion classifier (shape, gradient and option contracts)."""
import pytest
import torch

from complexity_framework_b200.generative import (IMUDeviceGraphTokenizer, SkeletonGraphTokenizer,
                                                  TRHashSensorFusionClassifier,
                                                  TRHashSensorFusionConfig, gradient_reverse)
from complexity_framework_b200.generative.sensor_structured import graph_adjacency


def test_encoders_keep_batch_and_token_shape_and_train():
    torch.manual_seed(0)
    sk = SkeletonGraphTokenizer(17, 3, hidden_size=64, token_count=8)
    imu = IMUDeviceGraphTokenizer(45, hidden_size=64, token_count=8)
    a, b = sk(torch.randn(2, 16, 17, 3)), imu(torch.randn(2, 16, 45))
    assert a.shape == (2, 8, 64) and b.shape == (2, 8, 64)
    (a.mean() + b.mean()).backward()
    assert sk.input_projection.weight.grad is not None
    assert imu.input_projection.weight.grad is not None
    assert sk.blocks[0].time_dw.weight.grad is not None


def test_encoders_reject_wrong_layouts():
    with pytest.raises(ValueError):
        SkeletonGraphTokenizer(25, 3, 64, 8)
    with pytest.raises(ValueError):
        IMUDeviceGraphTokenizer(44, 64, 8)
    with pytest.raises(ValueError):
        SkeletonGraphTokenizer(17, 3, 64, 8)(torch.randn(2, 16, 17, 2))


def test_adjacency_is_symmetric_normalised():
    a = graph_adjacency(5, IMUDeviceGraphTokenizer.EDGES)
    assert torch.allclose(a, a.T)
    # hub device 2 has degree 5 (four edges + self loop)
    assert torch.isclose(a[2, 2], torch.tensor(1 / 5))
    assert torch.isclose(a[0, 2], torch.tensor((1 / 2) ** 0.5 * (1 / 5) ** 0.5))


def test_gradient_reverse_flips_only_the_backward():
    v = torch.tensor([1.0, 2.0], requires_grad=True)
    out = gradient_reverse(v, 0.25)
    assert torch.equal(out, v)
    out.sum().backward()
    assert torch.allclose(v.grad, torch.full_like(v, -0.25))


def test_classifier_with_structured_encoders_and_subject_head():
    torch.manual_seed(0)
    cfg = TRHashSensorFusionConfig(num_classes=5, hidden_size=64, num_hidden_layers=1,
                                   num_attention_heads=4, num_experts=4, shared_width=64,
                                   expert_width=32, sequence_tokens=8, structured_encoders=True,
                                   num_subjects=3)
    m = TRHashSensorFusionClassifier(cfg)
    inputs = {"imu": torch.randn(2, 12, 45), "skeleton": torch.randn(2, 12, 17, 3)}
    out = m(inputs, labels=torch.tensor([1, 4]), subject_adversarial_scale=0.5)
    assert out["subject_logits"].shape == (2, 3)
    # the subject loss alone reaches the encoders with a reversed sign
    feats = out["features"]
    g_sub, = torch.autograd.grad(
        torch.nn.functional.cross_entropy(out["subject_logits"], torch.tensor([0, 2])),
        m.structured["imu"].input_projection.weight, retain_graph=True)
    assert torch.isfinite(g_sub).all() and g_sub.abs().sum() > 0
    out["loss"].backward()
    assert m.structured["skeleton"].input_projection.weight.grad is not None
    assert feats.shape == (2, 64)
    # default config keeps the flat projections
    plain = TRHashSensorFusionClassifier(TRHashSensorFusionConfig(
        num_classes=5, hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
        num_experts=4, shared_width=64, expert_width=32, sequence_tokens=8))
    assert not hasattr(plain, "structured") and "subject_logits" not in plain(inputs)


def _diag_model_and_batches():
    from complexity_framework_b200.generative.sensor_fusion import collate_sensors_masked

    torch.manual_seed(0)
    cfg = TRHashSensorFusionConfig(num_classes=4, hidden_size=64, num_hidden_layers=1,
                                   num_attention_heads=4, num_experts=4, shared_width=64,
                                   expert_width=32, sequence_tokens=8, classifier_dropout=0.0)
    m = TRHashSensorFusionClassifier(cfg)
    samples = [({"imu": torch.randn(12, 45), "skeleton": torch.randn(12, 17, 3)}, i % 4)
               for i in range(6)] + [({"imu": torch.randn(12, 45)}, 1), ({"imu": torch.randn(12, 45)}, 2)]
    batches = []
    for j in range(0, 8, 4):
        inputs, masks, labels = collate_sensors_masked(samples[j:j + 4])
        batches.append((inputs, masks, labels, torch.tensor([0, 0, 1, 1])))
    return m, batches


def test_sensor_diagnostics():
    from complexity_framework_b200.generative.sensor_diagnostics import (
        evaluate_late_fusion_sweep, evaluate_sensor_mode, hash_route_diagnostics)

    m, batches = _diag_model_and_batches()
    d = hash_route_diagnostics(m)["layers"]
    assert d and all(sum(v["expert_assignments"]) == v["routes"] * v["top_k"] for v in d.values())
    allm = evaluate_sensor_mode(m, batches, "cpu")
    assert allm["examples"] == 8 and set(allm["by_subject"]) == {"0", "1"}
    sk = evaluate_sensor_mode(m, batches, "cpu", modality="skeleton")
    assert sk["examples"] == 6 and sk["mode"] == "skeleton"
    sweep = evaluate_late_fusion_sweep(m, batches, "cpu", late_weights=(0.0, 1.0),
                                       gate_temperatures=(1.0,), stream_boosts={"skeleton": (1.0, 2.0)})
    assert len(sweep["results"]) == 4 and sweep["examples"] == 8
    # w = 1, T = 1, boost 1 is the model's own mixing (late_fusion_weight 0.5 =
    # (fused + per) / 2): same predictions as the plain evaluation
    own = next(r for r in sweep["results"] if r["late_weight"] == 1.0
               and r["boosts"] == {"skeleton": 1.0})
    assert own["accuracy"] == pytest.approx(allm["accuracy"])
    assert own["macro_f1"] == pytest.approx(allm["macro_f1"])
    with pytest.raises(ValueError):
        evaluate_late_fusion_sweep(m, batches, "cpu", gate_temperatures=(0.0,))
