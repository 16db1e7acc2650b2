"""TR-Hash vision / video towers (CPU): shapes, gradients, position routing."""
import torch

from complexity_framework_b200.generative.towers import (
    TRHashVideoClassifier, TRHashVideoTowerConfig, TRHashVisionClassifier, TRHashVisionTower,
    TRHashVisionTowerConfig)


def _vcfg(**kw):
    d = dict(image_size=32, patch_size=8, hidden_size=64, num_layers=2, num_heads=4,
             shared_width=128, expert_width=32)
    d.update(kw)
    return TRHashVisionTowerConfig(**d)


def test_vision_tower_and_classifier():
    torch.manual_seed(0)
    tower = TRHashVisionTower(_vcfg())
    x = torch.randn(2, 3, 32, 32)
    assert tower(x).shape == (2, 17, 64)
    assert tower.patch_features(x).shape == (2, 64, 4, 4)
    # patches route by position: every block's engine sees ids 0..P
    assert tower.route_ids.tolist() == [16] + list(range(16))
    clf = TRHashVisionClassifier(_vcfg(use_cls_token=False), 3)
    out = clf(x, torch.tensor([0, 2]))
    out["loss"].backward()
    assert out["logits"].shape == (2, 3)
    assert all(p.grad is not None for p in clf.parameters() if p.requires_grad)


def test_video_classifier_learns_a_batch():
    torch.manual_seed(0)
    cfg = TRHashVideoTowerConfig(image_size=32, patch_size=8, num_frames=4, hidden_size=64,
                                 num_layers=1, num_heads=4, shared_width=128, expert_width=32)
    m = TRHashVideoClassifier(cfg, 2)
    x = torch.randn(4, 3, 4, 32, 32)
    y = torch.tensor([0, 1, 0, 1])
    opt = torch.optim.AdamW(m.parameters(), 3e-3)
    first = None
    for _ in range(15):
        loss = m(x, y)["loss"]
        opt.zero_grad()
        loss.backward()
        opt.step()
        first = first if first is not None else float(loss)
    assert float(loss) < first
