"""Vision tasks on the TR-Hash tower (CPU): every task trains a step, fits a
tiny batch where it is cheap, and round-trips through its checkpoint."""
import math

import pytest
import torch

from complexity_framework_b200.generative.detection import TRHashDetectorConfig
from complexity_framework_b200.generative.vision_tasks import (
    SUPPORTED_VISION_TASKS, TRHashOBBDetector, TRHashPoseEstimator, create_vision_model,
    load_vision_task_checkpoint, save_vision_task_checkpoint)


def _cfg():
    return TRHashDetectorConfig(image_size=64, patch_size=16, hidden_size=64, num_layers=1,
                                num_heads=4, shared_width=128, expert_width=32, num_classes=3,
                                neck_channels=32)


def _batch(task):
    torch.manual_seed(0)
    x = torch.rand(2, 3, 64, 64)
    boxes = torch.tensor([[8., 8., 40., 36.]])
    if task in ("detection", "instance_segmentation"):
        m = torch.zeros(1, 64, 64)
        m[0, 8:36, 8:40] = 1
        return x, [{"boxes": boxes, "labels": torch.tensor([1]), "masks": m}] * 2
    if task == "obb":
        return x, [{"obb": torch.tensor([[30., 30., 30., 12., 0.5]]),
                    "labels": torch.tensor([2])}] * 2
    if task == "semantic_segmentation":
        return x, torch.randint(0, 3, (2, 64, 64))
    if task == "depth":
        return x, torch.rand(2, 64, 64) + 0.5
    if task == "classification":
        return x, torch.tensor([0, 2])
    kp = torch.tensor([[[10., 12., 1.], [40., 30., 1.], [0., 0., 0.]]]).repeat(2, 1, 1)
    return x, kp


@pytest.mark.parametrize("task", SUPPORTED_VISION_TASKS)
def test_task_trains_and_round_trips(task, tmp_path):
    torch.manual_seed(0)
    model = create_vision_model(task, _cfg(), num_keypoints=3, max_depth=4.0)
    x, y = _batch(task)
    opt = torch.optim.AdamW(model.parameters(), 2e-3)
    losses = []
    for _ in range(6):
        out = model(x, y)
        opt.zero_grad()
        out["loss"].backward()
        opt.step()
        losses.append(float(out["loss"]))
    assert all(math.isfinite(v) for v in losses)
    if task in ("semantic_segmentation", "depth", "classification", "pose"):
        assert losses[-1] < losses[0]
    if task == "instance_segmentation":
        assert "loss_mask" in out
    if task == "obb":
        assert "loss_angle" in out
    path = save_vision_task_checkpoint(model, str(tmp_path / task), task=task)
    back = load_vision_task_checkpoint(path)
    model.eval()
    a, b = model(x), back(x)
    key = next(k for k in ("logits", "depth", "heatmaps", "boxes") if k in a)
    assert torch.allclose(a[key], b[key], atol=1e-5)
    if task in ("detection", "instance_segmentation", "obb"):
        res = model.postprocess(model(x), score_threshold=0.0, max_detections=5)
        assert len(res) == 2
        if task == "instance_segmentation":
            assert res[0]["masks"].shape[0] == res[0]["boxes"].shape[0]
        if task == "obb":
            assert res[0]["obb"].shape == (res[0]["boxes"].shape[0], 5)


def test_obb_hull_and_pose_decode():
    obb = torch.tensor([[30., 20., 20., 10., 0.0], [30., 20., 20., 10., math.pi / 2]])
    h = TRHashOBBDetector.hull(obb)
    assert torch.allclose(h[0], torch.tensor([20., 15., 40., 25.]))
    assert torch.allclose(h[1], torch.tensor([25., 10., 35., 30.]), atol=1e-5)
    pose = TRHashPoseEstimator(_cfg(), num_keypoints=2)
    kp = torch.tensor([[[18., 30., 1.], [50., 6., 1.]]])
    dec = pose.decode(pose.heatmap_targets(kp, 64))
    assert torch.allclose(dec[0, :, :2], kp[0, :, :2], atol=2.0)
