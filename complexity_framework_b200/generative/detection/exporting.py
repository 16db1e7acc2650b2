"""Detector checkpoints and export.

Counterparts: complexity/generative/detection/checkpointing.py / exporting.py /
hub.py.  A checkpoint is ``config.json`` + ``model.pt`` (state dict) in a
directory; ``export_detector_torchscript`` traces the raw-output forward
(class logits and decoded boxes) for deployment runtimes.  ONNX / TensorRT
and hub upload need packages or network this framework does not assume.
"""
from __future__ import annotations

import json
import os

import torch

from .config import TRHashDetectorConfig
from .model import TRHashObjectDetector


def save_detector_checkpoint(model: TRHashObjectDetector, path: str, ema=None) -> None:
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(model.config.to_dict(), f, indent=2)
    sd = (ema.ema if ema is not None else model).state_dict()
    torch.save(sd, os.path.join(path, "model.pt"))


def load_detector_checkpoint(path: str, map_location="cpu") -> TRHashObjectDetector:
    with open(os.path.join(path, "config.json")) as f:
        cfg = TRHashDetectorConfig.from_dict(json.load(f))
    model = TRHashObjectDetector(cfg)
    model.load_state_dict(torch.load(os.path.join(path, "model.pt"), map_location=map_location))
    return model.eval()


class _RawOutputs(torch.nn.Module):
    def __init__(self, model: TRHashObjectDetector):
        super().__init__()
        self.model = model

    def forward(self, images: torch.Tensor):
        out = self.model(images)
        return out["cls_logits"].sigmoid(), out["boxes"]


def export_detector_torchscript(model: TRHashObjectDetector, path: str) -> str:
    """Trace (scores [B, A, C], boxes [B, A, 4]) and save; returns the file path."""
    model = model.eval()
    c = model.config
    example = torch.zeros(1, c.num_channels, c.image_size, c.image_size,
                          device=next(model.parameters()).device)
    with torch.no_grad():
        traced = torch.jit.trace(_RawOutputs(model), example, check_trace=False)
    traced.save(path)
    return path
