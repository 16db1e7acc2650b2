"""Box operations: IoU variants and non-maximum suppression (boxes are xyxy).

Counterparts: complexity/generative/detection/ops.py (``box_iou``,
``greedy_nms``, ``class_aware_nms``) and the CIoU term of losses.py.  NMS is a
vectorised greedy suppression: IoU matrix of the score-sorted boxes, then one
pass that keeps a box when no earlier kept box overlaps it above the
threshold (the same result as the classic loop).
"""
from __future__ import annotations

import math

import torch


def box_area(b: torch.Tensor) -> torch.Tensor:
    return (b[..., 2] - b[..., 0]).clamp_min(0) * (b[..., 3] - b[..., 1]).clamp_min(0)


def box_iou(a: torch.Tensor, b: torch.Tensor, eps: float = 1e-7) -> torch.Tensor:
    """[N, 4] x [M, 4] -> [N, M] IoU."""
    lt = torch.maximum(a[:, None, :2], b[None, :, :2])
    rb = torch.minimum(a[:, None, 2:], b[None, :, 2:])
    inter = (rb - lt).clamp_min(0).prod(-1)
    return inter / (box_area(a)[:, None] + box_area(b)[None, :] - inter + eps)


def complete_iou(a: torch.Tensor, b: torch.Tensor, eps: float = 1e-7) -> torch.Tensor:
    """Element-wise CIoU of matching rows of [..., 4] boxes (Zheng et al., 2020:
    IoU - centre distance^2 / enclosing diagonal^2 - alpha * v)."""
    lt = torch.maximum(a[..., :2], b[..., :2])
    rb = torch.minimum(a[..., 2:], b[..., 2:])
    inter = (rb - lt).clamp_min(0).prod(-1)
    union = box_area(a) + box_area(b) - inter + eps
    iou = inter / union
    c_lt = torch.minimum(a[..., :2], b[..., :2])
    c_rb = torch.maximum(a[..., 2:], b[..., 2:])
    c2 = ((c_rb - c_lt) ** 2).sum(-1) + eps
    ca = (a[..., :2] + a[..., 2:]) / 2
    cb = (b[..., :2] + b[..., 2:]) / 2
    rho2 = ((ca - cb) ** 2).sum(-1)
    wa, ha = (a[..., 2] - a[..., 0]).clamp_min(eps), (a[..., 3] - a[..., 1]).clamp_min(eps)
    wb, hb = (b[..., 2] - b[..., 0]).clamp_min(eps), (b[..., 3] - b[..., 1]).clamp_min(eps)
    v = (4 / math.pi ** 2) * (torch.atan(wb / hb) - torch.atan(wa / ha)) ** 2
    with torch.no_grad():
        alpha = v / (1 - iou + v + eps)
    return iou - rho2 / c2 - alpha * v


def complete_iou_loss(pred: torch.Tensor, target: torch.Tensor,
                      weight: torch.Tensor | None = None) -> torch.Tensor:
    loss = 1.0 - complete_iou(pred, target)
    if weight is not None:
        return (loss * weight).sum() / weight.sum().clamp_min(1e-6)
    return loss.mean()


def greedy_nms(boxes: torch.Tensor, scores: torch.Tensor, iou_threshold: float) -> torch.Tensor:
    """Indices (into ``boxes``) kept by greedy NMS, highest score first."""
    if boxes.numel() == 0:
        return torch.zeros(0, dtype=torch.long, device=boxes.device)
    order = scores.argsort(descending=True)
    b = boxes[order]
    over = box_iou(b, b) > iou_threshold
    n = b.shape[0]
    keep = torch.ones(n, dtype=torch.bool, device=boxes.device)
    over_cpu = over.cpu()
    keep_cpu = keep.cpu()
    for i in range(n):  # suppression is sequential by nature; the IoU matrix is not
        if keep_cpu[i]:
            keep_cpu[i + 1:] &= ~over_cpu[i, i + 1:]
    return order[keep_cpu.to(boxes.device)]


def class_aware_nms(boxes: torch.Tensor, scores: torch.Tensor, classes: torch.Tensor,
                    iou_threshold: float) -> torch.Tensor:
    """NMS within each class (boxes of different classes never suppress each other):
    boxes are offset by class so that cross-class IoU is zero."""
    if boxes.numel() == 0:
        return torch.zeros(0, dtype=torch.long, device=boxes.device)
    offset = classes.to(boxes.dtype)[:, None] * (boxes.max() + 1)
    return greedy_nms(boxes + offset, scores, iou_threshold)
