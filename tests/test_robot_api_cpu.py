"""Robot facade contract: the reference's config fields and [batch, channels,
time, height, width] clips build and run the sensor-fusion classifier
(claims of complexity/tests/test_robot_api.py)."""
import pytest
import torch

from complexity_framework_b200.api import Robot
from complexity_framework_b200.generative import (SENSOR_MODALITIES, TRHashSensorFusionClassifier,
                                                  TRHashSensorFusionConfig)


def _cfg(**over):
    kw = dict(hidden_size=32, num_hidden_layers=2, num_attention_heads=4, num_experts=8, top_k=2,
              shared_width=32, expert_width=8, precision="fp32", classifier_dropout=0.0,
              visual_channels=(3, 1, 3), visual_token_grid=(2, 2, 2), vision_image_size=16,
              vision_patch_size=4, vision_hidden_size=32, vision_layers=2, vision_heads=4,
              vision_num_experts=4, vision_top_k=2, vision_expert_width=8,
              vision_stage_depths=(1, 1), vision_window_size=2, radar_features=5,
              sequence_tokens=4)
    kw.update(over)
    return Robot.config(**kw)


def test_factory_builds_the_sensor_fusion_classifier():
    cfg = _cfg()
    m = Robot.from_config(cfg)
    assert isinstance(m, TRHashSensorFusionClassifier) and m.config == cfg
    assert Robot.MODALITIES == SENSOR_MODALITIES
    assert cfg.visual_layout == "bcthw" and cfg.visual_tokens == 8
    assert next(m.parameters()).dtype == torch.float32
    for blk in m.blocks:   # shared + sparse TR-Hash FFN in every block
        assert blk.mlp.config.shared_width > 0 and blk.mlp.config.expert_width > 0
        assert blk.mlp.config.top_k < blk.mlp.config.num_experts


def test_reference_layout_clips_and_sequences_run():
    torch.manual_seed(0)
    m = Robot.from_config(_cfg())
    B = 2
    out = m({"depth": torch.randn(B, 3, 4, 16, 16), "ir": torch.randn(B, 1, 4, 16, 16),
             "thermal": torch.randn(B, 3, 4, 16, 16), "imu": torch.randn(B, 12, 45),
             "radar": torch.randn(B, 10, 5), "skeleton": torch.randn(B, 8, 17, 3)},
            labels=torch.tensor([0, 1]))
    assert out["logits"].shape == (B, m.config.num_classes)
    out["loss"].backward()


def test_layouts_agree_on_the_same_clip():
    torch.manual_seed(0)
    a = TRHashSensorFusionClassifier(_cfg(visual_layout="btchw")).eval()
    b = TRHashSensorFusionClassifier(_cfg(visual_layout="bcthw")).eval()
    b.load_state_dict(a.state_dict())
    clip = torch.randn(2, 4, 3, 16, 16)                      # [B, T, C, H, W]
    ya = a({"depth": clip})["logits"]
    yb = b({"depth": clip.transpose(1, 2)})["logits"]        # [B, C, T, H, W]
    torch.testing.assert_close(ya, yb)


def test_config_validation():
    with pytest.raises(ValueError):
        _cfg(vision_stage_depths=(1, 2))
    with pytest.raises(ValueError):
        _cfg(visual_token_grid=(2, 2))
    with pytest.raises(ValueError):
        _cfg(precision="int4")
    assert Robot.from_config(_cfg(precision="bf16")).head.weight.dtype == torch.bfloat16
