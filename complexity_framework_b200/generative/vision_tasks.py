"""Dense and structured vision tasks on the TR-Hash vision tower.

Counterpart: complexity/generative/vision_tasks/ (``SUPPORTED_VISION_TASKS``,
``TRHashImageClassifier``, ``TRHashSemanticSegmenter``,
``TRHashDepthEstimator``, ``TRHashPoseEstimator``, ``TRHashInstanceSegmenter``,
``TRHashOBBDetector``, ``create_vision_model``, checkpoint save/load).  All
tasks take a ``TRHashDetectorConfig`` so one backbone configuration (and its
weights) moves between tasks.

* segmentation / depth / pose: tower feature map -> progressive 2x upsampling
  decoder -> per-pixel logits / depth / keypoint heatmaps;
* instance segmentation: the detector plus prototype masks (a small set of
  image-wide mask bases from the finest level) combined per detection with
  predicted coefficients, cropped to the box;
* oriented boxes: the detector plus a per-point angle, trained on the
  axis-aligned hull of each rotated box with an angle L1 term.
"""
from __future__ import annotations

import json
import math
import os
from typing import Dict, Literal, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .detection.config import TRHashDetectorConfig
from .detection.model import TRHashObjectDetector, _conv
from .towers import TRHashVisionTower, TRHashVisionTowerConfig

VisionTask = Literal["detection", "instance_segmentation", "semantic_segmentation", "depth",
                     "classification", "pose", "obb"]
SUPPORTED_VISION_TASKS = ("detection", "instance_segmentation", "semantic_segmentation",
                          "depth", "classification", "pose", "obb")


def _tower(c: TRHashDetectorConfig, cls_token: bool = False) -> TRHashVisionTower:
    return TRHashVisionTower(TRHashVisionTowerConfig(
        image_size=c.image_size, patch_size=c.patch_size, num_channels=c.num_channels,
        hidden_size=c.hidden_size, num_layers=c.num_layers, num_heads=c.num_heads,
        num_experts=c.num_experts, top_k=c.top_k, shared_width=c.shared_width,
        expert_width=c.expert_width, use_cls_token=cls_token))


class DenseDecoder(nn.Module):
    """Feature map at stride ``patch`` -> ``out_channels`` at stride ``final``
    through 2x upsampling stages."""

    def __init__(self, cin: int, channels: int, out_channels: int, patch: int, final: int = 1):
        super().__init__()
        stages = max(0, int(round(math.log2(patch // final))))
        layers = [_conv(cin, channels, 1)]
        for _ in range(stages):
            layers += [nn.Upsample(scale_factor=2.0, mode="bilinear", align_corners=False),
                       _conv(channels, channels)]
        self.body = nn.Sequential(*layers)
        self.out = nn.Conv2d(channels, out_channels, 1)

    def forward(self, x):
        return self.out(self.body(x))


class TRHashImageClassifier(nn.Module):
    def __init__(self, config: TRHashDetectorConfig, num_classes: Optional[int] = None):
        super().__init__()
        self.config = config
        self.tower = _tower(config, cls_token=True)
        self.head = nn.Linear(config.hidden_size, num_classes or config.num_classes)

    def forward(self, pixel_values, labels=None) -> Dict[str, torch.Tensor]:
        logits = self.head(self.tower(pixel_values)[:, 0])
        out = {"logits": logits}
        if labels is not None:
            out["loss"] = F.cross_entropy(logits.float(), labels)
        return out


class TRHashSemanticSegmenter(nn.Module):
    def __init__(self, config: TRHashDetectorConfig, num_classes: Optional[int] = None,
                 ignore_index: int = 255):
        super().__init__()
        self.config, self.ignore_index = config, ignore_index
        self.tower = _tower(config)
        self.decoder = DenseDecoder(config.hidden_size, config.neck_channels,
                                    num_classes or config.num_classes, config.patch_size, 4)

    def forward(self, pixel_values, labels=None) -> Dict[str, torch.Tensor]:
        """``labels`` [B, H, W] class ids (``ignore_index`` skipped)."""
        logits = F.interpolate(self.decoder(self.tower.patch_features(pixel_values)),
                               size=pixel_values.shape[-2:], mode="bilinear",
                               align_corners=False)
        out = {"logits": logits}
        if labels is not None:
            out["loss"] = F.cross_entropy(logits.float(), labels, ignore_index=self.ignore_index)
        return out


class TRHashDepthEstimator(nn.Module):
    """Per-pixel depth; trained with the scale-invariant log loss (Eigen et al.,
    2014, lambda 0.85) on pixels with positive ground truth."""

    def __init__(self, config: TRHashDetectorConfig, max_depth: Optional[float] = None):
        super().__init__()
        self.config, self.max_depth = config, max_depth
        self.tower = _tower(config)
        self.decoder = DenseDecoder(config.hidden_size, config.neck_channels, 1,
                                    config.patch_size, 4)

    def forward(self, pixel_values, depth=None) -> Dict[str, torch.Tensor]:
        x = F.interpolate(self.decoder(self.tower.patch_features(pixel_values)),
                          size=pixel_values.shape[-2:], mode="bilinear",
                          align_corners=False)[:, 0].float()
        pred = torch.sigmoid(x) * self.max_depth if self.max_depth else F.softplus(x) + 1e-3
        out = {"depth": pred}
        if depth is not None:
            m = depth > 0
            d = torch.log(pred[m].clamp_min(1e-6)) - torch.log(depth[m].float())
            out["loss"] = torch.sqrt((d ** 2).mean() - 0.85 * d.mean() ** 2 + 1e-8)
        return out


class TRHashPoseEstimator(nn.Module):
    """Keypoint heatmaps at stride 4; targets are Gaussians at visible keypoints."""

    def __init__(self, config: TRHashDetectorConfig, num_keypoints: int = 17, sigma: float = 2.0):
        super().__init__()
        self.config, self.K, self.sigma = config, num_keypoints, sigma
        self.tower = _tower(config)
        self.decoder = DenseDecoder(config.hidden_size, config.neck_channels, num_keypoints,
                                    config.patch_size, 4)

    def heatmap_targets(self, keypoints: torch.Tensor, size: int) -> torch.Tensor:
        """[B, K, 3] (x, y, visible) in pixels -> [B, K, size/4, size/4]."""
        h = size // 4
        ys, xs = torch.meshgrid(torch.arange(h, device=keypoints.device),
                                torch.arange(h, device=keypoints.device), indexing="ij")
        kx = keypoints[..., 0, None, None] / 4 - 0.5
        ky = keypoints[..., 1, None, None] / 4 - 0.5
        g = torch.exp(-((xs - kx) ** 2 + (ys - ky) ** 2) / (2 * self.sigma ** 2))
        return g * (keypoints[..., 2, None, None] > 0)

    def forward(self, pixel_values, keypoints=None) -> Dict[str, torch.Tensor]:
        hm = self.decoder(self.tower.patch_features(pixel_values)).float()
        out = {"heatmaps": hm, "keypoints": self.decode(hm)}
        if keypoints is not None:
            out["loss"] = F.mse_loss(hm, self.heatmap_targets(keypoints, pixel_values.shape[-1]))
        return out

    @staticmethod
    def decode(hm: torch.Tensor) -> torch.Tensor:
        """[B, K, h, w] -> [B, K, 3] (x, y, score) at the heatmap maxima, in pixels."""
        B, K, h, w = hm.shape
        score, idx = hm.flatten(2).max(-1)
        x = (idx % w).float() * 4 + 2
        y = (idx // w).float() * 4 + 2
        return torch.stack([x, y, score], -1)


class TRHashInstanceSegmenter(TRHashObjectDetector):
    """Detector + prototype masks: mask_i = sigmoid(coef_i . protos), cropped to
    box i.  Targets carry ``masks`` [n, H, W] (binary, image resolution)."""

    def __init__(self, config: TRHashDetectorConfig, num_prototypes: int = 16):
        super().__init__(config)
        C = config.neck_channels
        self.num_prototypes = num_prototypes
        self.protos = nn.Sequential(_conv(C, C), nn.Upsample(scale_factor=2.0, mode="nearest"),
                                    _conv(C, C), nn.Conv2d(C, num_prototypes, 1))
        self.coef = nn.Sequential(_conv(C, C), nn.Conv2d(C, num_prototypes, 1))

    def raw_outputs(self, feats):
        out = super().raw_outputs(feats)
        out["prototypes"] = self.protos(feats[0]).float()               # stride patch/4
        out["mask_coef"] = torch.cat([self.coef(f).flatten(2).transpose(1, 2) for f in feats],
                                     1).float()
        return out

    def _masks(self, protos: torch.Tensor, coef: torch.Tensor, boxes: torch.Tensor) -> torch.Tensor:
        """protos [P, h, w], coef [n, P], boxes [n, 4] (pixels) -> [n, h, w] logits, cropped."""
        h, w = protos.shape[-2:]
        logits = torch.einsum("np,phw->nhw", coef, protos)
        s = self.config.image_size / w
        xs = (torch.arange(w, device=protos.device) + 0.5) * s
        ys = (torch.arange(h, device=protos.device) + 0.5) * s
        inside = ((xs[None, None] >= boxes[:, 0, None, None]) & (xs[None, None] <= boxes[:, 2, None, None])
                  & (ys[None, :, None] >= boxes[:, 1, None, None]) & (ys[None, :, None] <= boxes[:, 3, None, None]))
        return logits.masked_fill(~inside, -20.0)

    def extra_loss_terms(self, out, b, target, fg, gidx, tval, acc) -> None:
        if "masks" not in target or not fg.any():
            return
        protos = out["prototypes"][b]
        h, w = protos.shape[-2:]
        gm = F.interpolate(target["masks"].to(protos.device, torch.float32)[None], size=(h, w),
                           mode="bilinear", align_corners=False)[0]
        tb = target["boxes"].to(protos.device, torch.float32)[gidx[fg]]
        pred = self._masks(protos, out["mask_coef"][b][fg], tb)
        loss = F.binary_cross_entropy_with_logits(pred, (gm[gidx[fg]] > 0.5).float())
        acc["loss_mask"] = acc.get("loss_mask", pred.new_zeros(())) + loss

    @torch.no_grad()
    def postprocess(self, out, **kw):
        res = super().postprocess(out, **kw)
        st = self.config.score_threshold if kw.get("score_threshold") is None else kw["score_threshold"]
        probs = out["cls_logits"].sigmoid()
        for b, r in enumerate(res):
            idx, lab = (probs[b] > st).nonzero(as_tuple=True)
            # recover each kept detection's point by matching its box and score
            cand_boxes = out["boxes"][b][idx].clamp(0, float(self.config.image_size))
            pts = []
            for bx in r["boxes"]:
                pts.append(int(idx[(cand_boxes - bx).abs().sum(-1).argmin()]))
            coef = out["mask_coef"][b][torch.tensor(pts, dtype=torch.long, device=idx.device)] \
                if pts else out["mask_coef"].new_zeros(0, self.num_prototypes)
            m = self._masks(out["prototypes"][b], coef, r["boxes"]).sigmoid()
            r["masks"] = F.interpolate(m[None], size=(self.config.image_size,) * 2,
                                       mode="bilinear", align_corners=False)[0] > 0.5 \
                if m.numel() else m.new_zeros(0, self.config.image_size, self.config.image_size,
                                              dtype=torch.bool)
        return res


class TRHashOBBDetector(TRHashObjectDetector):
    """Oriented boxes (cx, cy, w, h, angle in [-pi/4, 3pi/4)); targets carry
    ``obb`` [n, 5].  The box branch learns the axis-aligned hull; a per-point
    angle head adds the orientation."""

    def __init__(self, config: TRHashDetectorConfig):
        super().__init__(config)
        C = config.neck_channels
        self.angle = nn.Sequential(_conv(C, C), nn.Conv2d(C, 1, 1))

    @staticmethod
    def hull(obb: torch.Tensor) -> torch.Tensor:
        """[n, 5] rotated boxes -> [n, 4] axis-aligned xyxy hulls."""
        cx, cy, w, h, a = obb.unbind(-1)
        c, s = torch.cos(a).abs(), torch.sin(a).abs()
        hw, hh = (w * c + h * s) / 2, (w * s + h * c) / 2
        return torch.stack([cx - hw, cy - hh, cx + hw, cy + hh], -1)

    def raw_outputs(self, feats):
        out = super().raw_outputs(feats)
        a = torch.cat([self.angle(f).flatten(2).transpose(1, 2) for f in feats], 1).float()
        out["angles"] = (torch.sigmoid(a[..., 0]) - 0.25) * math.pi
        return out

    def loss(self, out, targets):
        hulls = [dict(t, boxes=self.hull(t["obb"].float())) if "obb" in t else t for t in targets]
        return super().loss(out, hulls)

    def extra_loss_terms(self, out, b, target, fg, gidx, tval, acc) -> None:
        if "obb" not in target or not fg.any():
            return
        ta = target["obb"].to(out["angles"].device, torch.float32)[gidx[fg], 4]
        d = out["angles"][b][fg] - ta
        d = torch.remainder(d + math.pi / 2, math.pi) - math.pi / 2  # angle period pi
        acc["loss_angle"] = acc.get("loss_angle", d.new_zeros(())) + F.smooth_l1_loss(
            d, torch.zeros_like(d), beta=0.1)

    @torch.no_grad()
    def postprocess(self, out, **kw):
        res = super().postprocess(out, **kw)
        st = self.config.score_threshold if kw.get("score_threshold") is None else kw["score_threshold"]
        probs = out["cls_logits"].sigmoid()
        for b, r in enumerate(res):
            idx, _ = (probs[b] > st).nonzero(as_tuple=True)
            cand = out["boxes"][b][idx].clamp(0, float(self.config.image_size))
            obb = []
            for bx in r["boxes"]:
                p = int(idx[(cand - bx).abs().sum(-1).argmin()])
                a = float(out["angles"][b][p])
                c, s = abs(math.cos(a)), abs(math.sin(a))
                W, H = float(bx[2] - bx[0]), float(bx[3] - bx[1])
                det = c * c - s * s
                if abs(det) > 1e-3:  # invert the hull: W = w c + h s, H = w s + h c
                    w, h = (W * c - H * s) / det, (H * c - W * s) / det
                else:
                    w = h = max(W, H) / (c + s)
                obb.append([float(bx[0] + bx[2]) / 2, float(bx[1] + bx[3]) / 2, abs(w), abs(h), a])
            r["obb"] = torch.tensor(obb, device=r["boxes"].device).reshape(-1, 5)
        return res


def create_vision_model(task: VisionTask, config: Optional[TRHashDetectorConfig] = None, *,
                        num_classes: Optional[int] = None, num_keypoints: int = 17,
                        num_prototypes: int = 16, max_depth: Optional[float] = None) -> nn.Module:
    if task not in SUPPORTED_VISION_TASKS:
        raise ValueError(f"unsupported vision task: {task}")
    config = config or TRHashDetectorConfig()
    if task == "detection":
        return TRHashObjectDetector(config)
    if task == "instance_segmentation":
        return TRHashInstanceSegmenter(config, num_prototypes)
    if task == "semantic_segmentation":
        return TRHashSemanticSegmenter(config, num_classes)
    if task == "depth":
        return TRHashDepthEstimator(config, max_depth)
    if task == "classification":
        return TRHashImageClassifier(config, num_classes)
    if task == "pose":
        return TRHashPoseEstimator(config, num_keypoints)
    return TRHashOBBDetector(config)


def save_vision_task_checkpoint(model: nn.Module, output: str, *, task: VisionTask,
                                class_names: Optional[Sequence[str]] = None) -> str:
    """Directory with ``vision_task.json`` (task, config, options, class names) and
    ``model.pt`` (state dict; loaded with ``weights_only``)."""
    if task not in SUPPORTED_VISION_TASKS:
        raise ValueError(f"unsupported vision task: {task}")
    os.makedirs(output, exist_ok=True)
    opts = {}
    if task == "instance_segmentation":
        opts["num_prototypes"] = model.num_prototypes
    if task == "depth":
        opts["max_depth"] = model.max_depth
    if task == "pose":
        opts["num_keypoints"] = model.K
    if task in ("semantic_segmentation",):
        opts["num_classes"] = model.decoder.out.out_channels
    if task == "classification":
        opts["num_classes"] = model.head.out_features
    manifest = {"format_version": 1, "task": task, "config": model.config.to_dict(),
                "options": opts, "class_names": list(class_names or model.config.class_names)}
    with open(os.path.join(output, "vision_task.json"), "w") as f:
        json.dump(manifest, f, indent=2)
    torch.save(model.state_dict(), os.path.join(output, "model.pt"))
    return output


def load_vision_task_checkpoint(checkpoint: str, *, device="cpu") -> nn.Module:
    with open(os.path.join(checkpoint, "vision_task.json")) as f:
        manifest = json.load(f)
    if manifest.get("format_version") != 1:
        raise ValueError("unsupported vision task checkpoint format")
    cfg = TRHashDetectorConfig.from_dict(manifest["config"])
    model = create_vision_model(manifest["task"], cfg, **manifest.get("options", {}))
    sd = torch.load(os.path.join(checkpoint, "model.pt"), map_location=device, weights_only=True)
    model.load_state_dict(sd, strict=True)
    return model.to(device).eval()
