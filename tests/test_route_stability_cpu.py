"""Fixed TR-Hash routes are part of every model's contract: two independent
constructions of the same config give identical route tables (so a
checkpoint's routes never depend on the RNG), and every table spreads its
routes over more than one expert."""
import pytest
import torch

from complexity_framework_b200 import ComplexityModel, ModelConfig
from complexity_framework_b200.generative import (TRHashSensorFusionClassifier,
                                                  TRHashSensorFusionConfig, TRHashVisionTower,
                                                  TRHashVisionTowerConfig)
from complexity_framework_b200.generative.detection import (TRHashDetectorConfig,
                                                            TRHashObjectDetector)

FACTORIES = {
    "decoder": lambda: ComplexityModel(ModelConfig(
        hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
        vocab_size=512, intermediate_size=64, shared_intermediate_size=128, num_experts=4,
        top_k=2, max_position_embeddings=128)),
    "vision_tower": lambda: TRHashVisionTower(TRHashVisionTowerConfig(
        image_size=32, patch_size=8, hidden_size=64, num_layers=2, num_heads=4,
        shared_width=64, expert_width=16)),
    "sensor_fusion": lambda: TRHashSensorFusionClassifier(TRHashSensorFusionConfig(
        num_classes=4, hidden_size=64, num_hidden_layers=1, num_attention_heads=4,
        num_experts=4, shared_width=64, expert_width=16, sequence_tokens=8)),
    "detector": lambda: TRHashObjectDetector(TRHashDetectorConfig(
        image_size=64, patch_size=16, hidden_size=64, num_layers=1, num_heads=4,
        shared_width=128, expert_width=32, num_classes=2, neck_channels=32)),
}


def _tables(model):
    return {n: b.detach().clone() for n, b in model.named_buffers() if n.endswith("route_table")}


@pytest.mark.parametrize("name", sorted(FACTORIES))
def test_route_tables_are_deterministic_and_spread(name):
    torch.manual_seed(1)
    a = _tables(FACTORIES[name]())
    torch.manual_seed(2)          # a different RNG state must not change routes
    b = _tables(FACTORIES[name]())
    assert a, f"{name}: no route table"
    assert set(a) == set(b)
    for k in a:
        assert torch.equal(a[k], b[k]), f"{name}:{k} differs between constructions"
        assert torch.unique(a[k]).numel() > 1, f"{name}:{k} routes to a single expert"
