"""``TRHashObjectDetector``: anchor-free multi-scale detector on the TR-Hash
vision tower.

Counterpart: complexity/generative/detection/model.py / head.py /
hierarchical_tower.py / targets.py.  Structure here: the TR-Hash tower gives a
stride-``patch`` feature map; a small neck derives stride patch/2 (upsampled)
and 2*patch (strided conv) levels; a decoupled head shared across levels
predicts per-point class logits and, per box side, a distribution over
``reg_max`` distance bins (decoded as its expectation, in stride units).
Training assigns objects to points with a task-aligned rule (candidate points
inside the box, top-k by score^alpha * IoU^beta, ties to the highest IoU) and
uses quality focal loss (IoU-valued class targets), CIoU and distribution
focal loss.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..towers import TRHashVisionTower, TRHashVisionTowerConfig
from .config import TRHashDetectorConfig
from .losses import distribution_focal_loss, quality_focal_loss
from .ops import box_iou, class_aware_nms, complete_iou


def _conv(cin: int, cout: int, k: int = 3, s: int = 1) -> nn.Sequential:
    return nn.Sequential(nn.Conv2d(cin, cout, k, s, k // 2, bias=False), nn.GroupNorm(8, cout),
                         nn.SiLU())


class DetectionHead(nn.Module):
    def __init__(self, channels: int, num_classes: int, reg_max: int):
        super().__init__()
        self.cls = nn.Sequential(_conv(channels, channels), _conv(channels, channels),
                                 nn.Conv2d(channels, num_classes, 1))
        self.reg = nn.Sequential(_conv(channels, channels), _conv(channels, channels),
                                 nn.Conv2d(channels, 4 * reg_max, 1))
        nn.init.constant_(self.cls[-1].bias, -4.6)  # prior probability ~1 %

    def forward(self, x):
        return self.cls(x), self.reg(x)


class TRHashObjectDetector(nn.Module):
    def __init__(self, config: TRHashDetectorConfig):
        super().__init__()
        self.config = c = config
        C = c.neck_channels
        if c.backbone == "hierarchical":
            from ..hierarchical import HierarchicalTowerConfig, HierarchicalTRHashVisionTower

            self.tower = HierarchicalTRHashVisionTower(HierarchicalTowerConfig(
                image_size=c.image_size, num_channels=c.num_channels, dims=c.hier_dims,
                depths=c.hier_depths, heads=c.hier_heads, window_size=c.hier_window,
                num_experts=c.num_experts, top_k=c.top_k))
            # top-down pyramid over the stride 8 / 16 / 32 stage maps
            self.laterals = nn.ModuleList(_conv(d, C, 1) for d in c.hier_dims[1:4])
            self.smooth = nn.ModuleList(_conv(C, C) for _ in range(3))
            self.head = DetectionHead(C, c.num_classes, c.reg_max)
            self.register_buffer("bins", torch.arange(c.reg_max, dtype=torch.float32),
                                 persistent=False)
            return
        self.tower = TRHashVisionTower(TRHashVisionTowerConfig(
            image_size=c.image_size, patch_size=c.patch_size, num_channels=c.num_channels,
            hidden_size=c.hidden_size, num_layers=c.num_layers, num_heads=c.num_heads,
            num_experts=c.num_experts, top_k=c.top_k, shared_width=c.shared_width,
            expert_width=c.expert_width, use_cls_token=False))
        self.lateral = _conv(c.hidden_size, C, 1)
        self.up = _conv(C, C)
        self.down = _conv(C, C, 3, 2)
        self.head = DetectionHead(C, c.num_classes, c.reg_max)
        self.register_buffer("bins", torch.arange(c.reg_max, dtype=torch.float32),
                             persistent=False)

    # --------------------------------------------------------------- forward
    def features(self, images: torch.Tensor) -> List[torch.Tensor]:
        if self.config.backbone == "hierarchical":
            s8, s16, s32 = self.tower(images)[1:4]
            p5 = self.laterals[2](s32)
            p4 = self.laterals[1](s16) + F.interpolate(p5, size=s16.shape[-2:], mode="nearest")
            p3 = self.laterals[0](s8) + F.interpolate(p4, size=s8.shape[-2:], mode="nearest")
            return [self.smooth[0](p3), self.smooth[1](p4), self.smooth[2](p5)]
        p4 = self.lateral(self.tower.patch_features(images))
        p3 = self.up(F.interpolate(p4, scale_factor=2.0, mode="nearest"))
        p5 = self.down(p4)
        return [p3, p4, p5]

    def anchors(self, feats: List[torch.Tensor]):
        pts, strides = [], []
        for f, s in zip(feats, self.config.strides):
            h, w = f.shape[-2:]
            ys, xs = torch.meshgrid(torch.arange(h, device=f.device),
                                    torch.arange(w, device=f.device), indexing="ij")
            p = torch.stack([xs, ys], -1).reshape(-1, 2).float() + 0.5
            pts.append(p * s)
            strides.append(torch.full((h * w,), float(s), device=f.device))
        return torch.cat(pts), torch.cat(strides)

    def forward(self, images: torch.Tensor,
                targets: Optional[List[Dict[str, torch.Tensor]]] = None) -> Dict:
        out = self.raw_outputs(self.features(images))
        if targets is not None:
            out.update(self.loss(out, targets))
        return out

    def raw_outputs(self, feats: List[torch.Tensor]) -> Dict:
        """Per-point class logits, box distributions and decoded boxes of all levels."""
        cls, reg = [], []
        for f in feats:
            c, r = self.head(f)
            cls.append(c.flatten(2).transpose(1, 2))
            reg.append(r.flatten(2).transpose(1, 2))
        cls = torch.cat(cls, 1).float()                              # [B, A, C]
        reg = torch.cat(reg, 1).float()                              # [B, A, 4 * bins]
        points, strides = self.anchors(feats)
        B, A = cls.shape[:2]
        dist = reg.view(B, A, 4, self.config.reg_max)
        ltrb = (dist.softmax(-1) * self.bins).sum(-1) * strides[None, :, None]
        boxes = torch.cat([points - ltrb[..., :2], points + ltrb[..., 2:]], -1)
        return {"cls_logits": cls, "box_dist": dist, "boxes": boxes, "points": points,
                "strides": strides, "features": feats}

    # ------------------------------------------------------------ assignment
    @torch.no_grad()
    def assign(self, scores, boxes, points, gt_boxes, gt_labels):
        """Per image: (fg mask [A], target boxes [A, 4], target labels [A], soft
        class-target values [A], matched object index [A])."""
        c = self.config
        A = points.shape[0]
        dev = points.device
        fg = torch.zeros(A, dtype=torch.bool, device=dev)
        tbox = torch.zeros(A, 4, device=dev)
        tlab = torch.zeros(A, dtype=torch.long, device=dev)
        tval = torch.zeros(A, device=dev)
        if gt_boxes.numel() == 0:
            return fg, tbox, tlab, tval, torch.zeros(A, dtype=torch.long, device=dev)
        inside = ((points[None, :, 0] > gt_boxes[:, None, 0]) & (points[None, :, 0] < gt_boxes[:, None, 2])
                  & (points[None, :, 1] > gt_boxes[:, None, 1]) & (points[None, :, 1] < gt_boxes[:, None, 3]))
        iou = box_iou(gt_boxes, boxes).clamp_min(0)                  # [G, A]
        sc = scores[:, gt_labels].T                                   # [G, A]
        align = sc.pow(c.assign_alpha) * iou.pow(c.assign_beta) * inside
        k = min(c.assign_topk, A)
        top = align.topk(k, dim=1).indices
        cand = torch.zeros_like(inside)
        cand.scatter_(1, top, True)
        cand &= inside
        # an object with no point inside it (tiny box) takes its nearest point
        none = ~cand.any(1)
        if none.any():
            ctr = (gt_boxes[none, :2] + gt_boxes[none, 2:]) / 2
            near = torch.cdist(ctr, points).argmin(1)
            cand[none.nonzero().squeeze(1), near] = True
        iou_c = torch.where(cand, iou, torch.full_like(iou, -1.0))
        g = iou_c.argmax(0)                                           # best object per point
        fg = cand.any(0)
        tbox = gt_boxes[g]
        tlab = gt_labels[g]
        align = align * cand
        norm = align / align.amax(1, keepdim=True).clamp_min(1e-9) * (iou * cand).amax(1, keepdim=True)
        tval = norm.gather(0, g[None]).squeeze(0) * fg
        return fg, tbox, tlab, tval, g

    def loss(self, out: Dict, targets: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
        c = self.config
        cls, dist, boxes = out["cls_logits"], out["box_dist"], out["boxes"]
        points, strides = out["points"], out["strides"]
        scores = cls.detach().sigmoid()
        l_cls, l_box, l_dfl, norm = cls.new_zeros(()), cls.new_zeros(()), cls.new_zeros(()), 0.0
        parts_extra: Dict[str, torch.Tensor] = {}
        for b, t in enumerate(targets):
            gb = t["boxes"].to(boxes.device, torch.float32)
            gl = t["labels"].to(boxes.device, torch.long)
            fg, tbox, tlab, tval, gidx = self.assign(scores[b], boxes[b].detach(), points, gb, gl)
            self.extra_loss_terms(out, b, t, fg, gidx, tval, parts_extra)
            target = torch.zeros_like(cls[b])
            if fg.any():
                target[fg, tlab[fg]] = tval[fg]
            l_cls = l_cls + quality_focal_loss(cls[b], target)
            norm += float(tval.sum())
            if fg.any():
                w = tval[fg]
                l_box = l_box + ((1.0 - complete_iou(boxes[b][fg], tbox[fg])) * w).sum()
                s = strides[fg][:, None]
                p = points[fg]
                ltrb = torch.cat([p - tbox[fg, :2], tbox[fg, 2:] - p], -1) / s
                dfl = distribution_focal_loss(dist[b][fg].reshape(-1, c.reg_max),
                                              ltrb.reshape(-1)).view(-1, 4).mean(-1)
                l_dfl = l_dfl + (dfl * w).sum()
        norm = max(norm, 1.0)
        wc, wb, wd = c.loss_weights
        parts = {"loss_cls": l_cls / norm, "loss_box": l_box / norm, "loss_dfl": l_dfl / norm}
        parts["loss"] = wc * parts["loss_cls"] + wb * parts["loss_box"] + wd * parts["loss_dfl"]
        for k, v in parts_extra.items():  # task heads of subclasses (masks, angles)
            parts[k] = v / len(targets)
            parts["loss"] = parts["loss"] + parts[k]
        return parts

    def extra_loss_terms(self, out, b, target, fg, gidx, tval, acc) -> None:
        """Hook for task heads built on the detector: add per-image loss terms to
        ``acc`` (summed over images, divided by the batch size)."""

    # ---------------------------------------------------------- postprocess
    @torch.no_grad()
    def postprocess(self, out: Dict, score_threshold: Optional[float] = None,
                    iou_threshold: Optional[float] = None,
                    max_detections: Optional[int] = None) -> List[Dict[str, torch.Tensor]]:
        c = self.config
        st = c.score_threshold if score_threshold is None else score_threshold
        it = c.nms_iou if iou_threshold is None else iou_threshold
        md = c.max_detections if max_detections is None else max_detections
        res = []
        probs = out["cls_logits"].sigmoid()
        size = float(c.image_size)
        for b in range(probs.shape[0]):
            p = probs[b]
            idx, lab = (p > st).nonzero(as_tuple=True)
            sc = p[idx, lab]
            bx = out["boxes"][b][idx].clamp(0, size)
            if sc.numel() > 4096:  # NMS builds a dense IoU matrix of the candidates
                top = sc.topk(4096).indices
                idx, lab, sc, bx = idx[top], lab[top], sc[top], bx[top]
            keep = class_aware_nms(bx, sc, lab, it)[:md]
            res.append({"boxes": bx[keep], "scores": sc[keep], "labels": lab[keep]})
        return res

    @torch.no_grad()
    def predict(self, images: torch.Tensor, **kw) -> List[Dict[str, torch.Tensor]]:
        was = self.training
        self.eval()
        try:
            return self.postprocess(self.forward(images), **kw)
        finally:
            self.train(was)
