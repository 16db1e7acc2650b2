"""Detector configuration (counterpart: complexity/generative/detection/config.py
``TRHashDetectorConfig`` and presets.py ``coco_v8_nano_config``)."""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Tuple


@dataclass
class TRHashDetectorConfig:
    image_size: int = 320
    patch_size: int = 16
    num_channels: int = 3
    hidden_size: int = 192
    num_layers: int = 4
    num_heads: int = 6
    num_experts: int = 4
    top_k: int = 2
    shared_width: int = 384
    expert_width: int = 64
    num_classes: int = 80
    neck_channels: int = 128
    reg_max: int = 16                  # distribution bins per box side (DFL)
    # task-aligned assignment (score^alpha * IoU^beta, top-k candidates per object)
    assign_topk: int = 10
    assign_alpha: float = 0.5
    assign_beta: float = 6.0
    loss_weights: Tuple[float, float, float] = (1.0, 7.5, 1.5)  # cls, box (CIoU), dfl
    score_threshold: float = 0.05
    nms_iou: float = 0.6
    max_detections: int = 300
    class_names: Tuple[str, ...] = field(default_factory=tuple)
    # "plain": one ViT-style tower at stride patch_size with a derived pyramid;
    # "hierarchical": the windowed multi-stage tower (real stride 8/16/32 maps)
    backbone: str = "plain"
    hier_dims: Tuple[int, ...] = (64, 128, 256, 384)
    hier_depths: Tuple[int, ...] = (1, 1, 2, 1)
    hier_heads: Tuple[int, ...] = (2, 4, 8, 12)
    hier_window: int = 8

    def __post_init__(self):
        if self.backbone not in ("plain", "hierarchical"):
            raise ValueError("backbone must be 'plain' or 'hierarchical'")
        if self.backbone == "plain" and self.image_size % (2 * self.patch_size):
            raise ValueError("image_size must be a multiple of 2 * patch_size")
        if self.backbone == "hierarchical" and self.image_size % 32:
            raise ValueError("the hierarchical backbone needs image_size % 32 == 0")

    @property
    def strides(self) -> Tuple[int, int, int]:
        if self.backbone == "hierarchical":
            return (8, 16, 32)
        return (self.patch_size // 2, self.patch_size, self.patch_size * 2)

    def to_dict(self) -> dict:
        d = asdict(self)
        for k in ("class_names", "loss_weights", "hier_dims", "hier_depths", "hier_heads"):
            d[k] = list(d[k])
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "TRHashDetectorConfig":
        d = dict(d)
        d["class_names"] = tuple(d.get("class_names", ()))
        d["loss_weights"] = tuple(d.get("loss_weights", (1.0, 7.5, 1.5)))
        for k in ("hier_dims", "hier_depths", "hier_heads"):
            if k in d:
                d[k] = tuple(d[k])
        return cls(**d)


COCO_V8_NANO_NAME = "tr-hash-det-coco-nano"


def coco_v8_nano_config(**overrides) -> TRHashDetectorConfig:
    """Small COCO preset (80 classes, 640 px input)."""
    from .data import COCO_CLASS_NAMES

    base = dict(image_size=640, patch_size=16, hidden_size=256, num_layers=6, num_heads=8,
                shared_width=512, expert_width=96, num_classes=80, neck_channels=128,
                class_names=tuple(COCO_CLASS_NAMES))
    base.update(overrides)
    return TRHashDetectorConfig(**base)
