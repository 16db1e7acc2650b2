"""COCO-style detection metrics: AP at IoU 0.50:0.95, object-size buckets, and
fixed-confidence / best-F1 operating points, accumulated image by image and
mergeable across ranks.

Counterpart of complexity/generative/detection/metrics.py:10-265
(``DetectionMetricsAccumulator``): the same IoU thresholds, COCO area ranges
(small < 32^2 <= medium < 96^2 <= large pixels), greedy score-ordered matching
and all-point interpolated AP, and the same result keys (map50, map50_95,
precision, recall, f1, best_f1, best_confidence, ap_small/medium/large).

Matching is done once per (image, class) for all ten thresholds together: the
IoU matrix of the score-sorted predictions against the ground truth is
computed once and, walking the predictions in order, each threshold takes the
best still-free ground-truth box whose IoU clears it.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

IOU_THRESHOLDS = tuple(round(0.50 + 0.05 * i, 2) for i in range(10))
SIZE_RANGES = {"small": (0.0, 32.0 ** 2), "medium": (32.0 ** 2, 96.0 ** 2),
               "large": (96.0 ** 2, float("inf"))}
SCOPES = ("all",) + tuple(SIZE_RANGES)


def cxcywh_to_xyxy(b: torch.Tensor) -> torch.Tensor:
    return torch.cat((b[:, :2] - b[:, 2:4] / 2, b[:, :2] + b[:, 2:4] / 2), -1)


def _areas(b: torch.Tensor) -> torch.Tensor:
    return (b[:, 2:] - b[:, :2]).clamp_min(0).prod(-1)


def _pair_iou(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if not len(a) or not len(b):
        return torch.zeros(len(a), len(b))
    lt = torch.maximum(a[:, None, :2], b[None, :, :2])
    rb = torch.minimum(a[:, None, 2:], b[None, :, 2:])
    inter = (rb - lt).clamp_min(0).prod(-1)
    return inter / (_areas(a)[:, None] + _areas(b)[None] - inter).clamp_min(1e-9)


def greedy_match(boxes: torch.Tensor, scores: torch.Tensor, gt: torch.Tensor):
    """(sorted scores [P], matched [T, P] bool) for the IoU thresholds T."""
    order = torch.argsort(scores, descending=True)
    scores, boxes = scores[order], boxes[order]
    T = len(IOU_THRESHOLDS)
    matched = torch.zeros(T, len(boxes), dtype=torch.bool)
    if len(gt) and len(boxes):
        iou = _pair_iou(boxes, gt)
        thr = torch.tensor(IOU_THRESHOLDS)[:, None]
        free = torch.ones(T, len(gt), dtype=torch.bool)
        for p in torch.nonzero((iou >= IOU_THRESHOLDS[0]).any(1)).flatten().tolist():
            cand = iou[p][None].expand(T, -1).masked_fill(~free, -1.0)
            best, j = cand.max(1)
            ok = best >= thr[:, 0]
            matched[ok, p] = True
            free[ok, j[ok]] = False
    return scores, matched


def average_precision(scores: torch.Tensor, tp: torch.Tensor, n_gt: int) -> float:
    """All-point interpolated AP (NaN when the class has no ground truth)."""
    if n_gt == 0:
        return float("nan")
    if not len(scores):
        return 0.0
    tp = tp[torch.argsort(scores, descending=True)].float()
    ctp = tp.cumsum(0)
    recall = torch.cat((torch.zeros(1), ctp / n_gt, torch.ones(1)))
    prec = torch.cat((torch.ones(1), ctp / torch.arange(1, len(tp) + 1), torch.zeros(1)))
    prec = prec.flip(0).cummax(0).values.flip(0)
    step = torch.nonzero(recall[1:] != recall[:-1]).flatten()
    return float(((recall[step + 1] - recall[step]) * prec[step + 1]).sum())


class DetectionMetricsAccumulator:
    """Per (scope, class): the predictions' scores, their matches at every IoU
    threshold, and the ground-truth count.  ``image_size`` converts normalised
    boxes to pixels for the size buckets (1 when boxes are already in pixels)."""

    def __init__(self, num_classes: int, image_size: int = 1):
        self.num_classes, self.image_size = num_classes, image_size
        self._scores = {s: [[] for _ in range(num_classes)] for s in SCOPES}
        self._matches = {s: [[] for _ in range(num_classes)] for s in SCOPES}
        self._gt = {s: [0] * num_classes for s in SCOPES}

    def update(self, boxes: torch.Tensor, scores: torch.Tensor, labels: torch.Tensor,
               targets: torch.Tensor) -> None:
        """Reference format: predictions as normalised xyxy, targets [N, 5] rows
        (cx, cy, w, h, label) normalised."""
        t = targets.float().cpu()
        self.update_xyxy(boxes, scores, labels, cxcywh_to_xyxy(t[:, :4]), t[:, 4].long())

    def update_xyxy(self, boxes: torch.Tensor, scores: torch.Tensor, labels: torch.Tensor,
                    gt_boxes: torch.Tensor, gt_labels: torch.Tensor) -> None:
        """One image: predictions and ground truth as xyxy in the same units."""
        boxes, scores = boxes.float().cpu(), scores.float().cpu()
        labels, gt_boxes, gt_labels = labels.long().cpu(), gt_boxes.float().cpu(), gt_labels.long().cpu()
        px = float(self.image_size) ** 2
        pa, ga = _areas(boxes) * px, _areas(gt_boxes) * px
        masks = {"all": (torch.ones(len(boxes), dtype=torch.bool),
                         torch.ones(len(gt_boxes), dtype=torch.bool))}
        for name, (lo, hi) in SIZE_RANGES.items():
            masks[name] = ((pa >= lo) & (pa < hi), (ga >= lo) & (ga < hi))
        for c in range(self.num_classes):
            pc, gc = labels == c, gt_labels == c
            for scope, (pm, gm) in masks.items():
                p, g = pc & pm, gc & gm
                s, m = greedy_match(boxes[p], scores[p], gt_boxes[g])
                self._scores[scope][c].append(s)
                self._matches[scope][c].append(m)
                self._gt[scope][c] += int(g.sum())

    # ---------------------------------------------------- cross-rank merge
    def state_dict(self) -> Dict:
        cat = self._cat
        return {"scores": {s: [cat(v) for v in self._scores[s]] for s in SCOPES},
                "matches": {s: [cat(v, 2) for v in self._matches[s]] for s in SCOPES},
                "target_counts": {s: list(self._gt[s]) for s in SCOPES}}

    def merge_state_dict(self, state: Dict) -> None:
        for s in SCOPES:
            for c in range(self.num_classes):
                self._scores[s][c].append(state["scores"][s][c])
                self._matches[s][c].append(state["matches"][s][c])
                self._gt[s][c] += int(state["target_counts"][s][c])

    @staticmethod
    def _cat(values: List[torch.Tensor], dims: int = 1) -> torch.Tensor:
        if values:
            return torch.cat(values, -1)
        return torch.empty(0) if dims == 1 else torch.zeros(len(IOU_THRESHOLDS), 0,
                                                            dtype=torch.bool)

    # ----------------------------------------------------------- results
    def _map(self, scope: str, t: int) -> float:
        aps = [average_precision(self._cat(self._scores[scope][c]),
                                 self._cat(self._matches[scope][c], 2)[t], self._gt[scope][c])
               for c in range(self.num_classes)]
        aps = [a for a in aps if not math.isnan(a)]
        return sum(aps) / max(len(aps), 1)

    def compute(self, confidence_threshold: float = 0.25) -> Dict[str, float]:
        T = len(IOU_THRESHOLDS)
        per_t = [self._map("all", t) for t in range(T)]
        sc = torch.cat([self._cat(v) for v in self._scores["all"]])
        mt = torch.cat([self._cat(v, 2)[0] for v in self._matches["all"]]).float()
        order = torch.argsort(sc, descending=True)
        sc, mt = sc[order], mt[order]
        n_gt = sum(self._gt["all"])
        keep = sc >= confidence_threshold
        tp = float(mt[keep].sum())
        precision, recall = tp / max(int(keep.sum()), 1), tp / max(n_gt, 1)
        f1 = 2 * precision * recall / max(precision + recall, 1e-9)
        if len(sc):
            curve = 2 * mt.cumsum(0) / (torch.arange(1, len(sc) + 1) + n_gt).clamp_min(1)
            best, i = curve.max(0)
            best_f1, best_conf = float(best), float(sc[int(i)])
        else:
            best_f1, best_conf = 0.0, 1.0
        out = {"map50": per_t[0], "map50_95": sum(per_t) / T, "precision": precision,
               "recall": recall, "f1": f1, "best_f1": best_f1, "best_confidence": best_conf}
        for name in SIZE_RANGES:
            out[f"ap_{name}"] = sum(self._map(name, t) for t in range(T)) / T
        return out


def evaluate_predictions(predictions, targets, num_classes: int,
                         confidence_threshold: float = 0.25,
                         accumulator: Optional[DetectionMetricsAccumulator] = None
                         ) -> Dict[str, float]:
    """Score lists of per-image prediction dicts (boxes xyxy pixels, scores,
    labels) against target dicts (boxes, labels) in the same pixel units."""
    acc = accumulator or DetectionMetricsAccumulator(num_classes)
    for p, t in zip(predictions, targets):
        acc.update_xyxy(p["boxes"], p["scores"], p["labels"], t["boxes"], t["labels"])
    return acc.compute(confidence_threshold)
