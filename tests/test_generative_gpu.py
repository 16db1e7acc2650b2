"""Generative models on a B200: the TR-Hash feed-forwards of the vision tower
and the detector run the fused sm_100a path in bf16 and agree with the fp32
PyTorch path on the same weights."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_vision_tower_fused_matches_fp32():
    from complexity_framework_b200.generative.towers import (TRHashVisionTower,
                                                             TRHashVisionTowerConfig)
    from complexity_framework_b200.tr_hash.config import TRHashBackend

    torch.manual_seed(0)
    cfg = TRHashVisionTowerConfig(image_size=128, patch_size=16, hidden_size=256, num_layers=2,
                                  num_heads=4, shared_width=512, expert_width=64)
    ref = TRHashVisionTower(cfg).cuda().float()
    fast = copy.deepcopy(ref).to(torch.bfloat16)
    x = torch.randn(4, 3, 128, 128, device="cuda")
    y_ref = ref(x)
    y = fast(x.bfloat16())
    assert all(b.mlp.last_backend.selected is TRHashBackend.FUSED_CUDA for b in fast.blocks)
    rel = float((y.float() - y_ref).norm() / y_ref.norm())
    assert rel < 3e-2, rel
    y.float().square().mean().backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all()
               for p in fast.parameters() if p.requires_grad)


def test_detector_trains_in_bf16_on_gpu():
    from complexity_framework_b200.generative.detection import (
        DetectorTrainer, DetectorTrainingConfig, SyntheticShapesDataset, TRHashDetectorConfig,
        TRHashObjectDetector, collate_detection)

    torch.manual_seed(0)
    cfg = TRHashDetectorConfig(image_size=128, patch_size=16, hidden_size=256, num_layers=2,
                               num_heads=4, shared_width=512, expert_width=64, num_classes=2,
                               neck_channels=64)
    m = TRHashObjectDetector(cfg).cuda()
    dl = torch.utils.data.DataLoader(SyntheticShapesDataset(64, 128, 3, 2), batch_size=16,
                                     collate_fn=collate_detection)
    ev = torch.utils.data.DataLoader(SyntheticShapesDataset(32, 128, 3, 2, seed=5),
                                     batch_size=16, collate_fn=collate_detection)
    tr = DetectorTrainer(m, DetectorTrainingConfig(learning_rate=2e-3, warmup_steps=10,
                                                   max_steps=60, ema_tau=10))
    for _ in range(12):
        for im, tg in dl:
            tr.train_step(im, tg)
    assert tr.evaluate(ev, use_ema=False)["AP50"] > 0.3


def test_autocast_uses_fused_tr_hash_path():
    """Generative blocks trained under bf16 autocast feed the TR-Hash engine bf16."""
    from complexity_framework_b200.generative.towers import (TRHashVisionClassifier,
                                                             TRHashVisionTowerConfig)
    from complexity_framework_b200.tr_hash.config import TRHashBackend

    torch.manual_seed(0)
    cfg = TRHashVisionTowerConfig(image_size=64, patch_size=16, hidden_size=256, num_layers=1,
                                  num_heads=4, shared_width=512, expert_width=64)
    m = TRHashVisionClassifier(cfg, 4).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = m(torch.randn(8, 3, 64, 64, device="cuda"), torch.randint(0, 4, (8,), device="cuda"))
    out["loss"].backward()
    assert m.tower.blocks[0].mlp.last_backend.selected is TRHashBackend.FUSED_CUDA
    assert torch.isfinite(m.tower.patch.weight.grad).all()
