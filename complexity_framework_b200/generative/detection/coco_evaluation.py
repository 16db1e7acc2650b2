"""COCO-style detection metrics computed in-process.

Counterpart: complexity/generative/detection/coco_evaluation.py (which calls
pycocotools).  Same protocol: per class, detections sorted by score are
greedily matched to unmatched ground truth of IoU >= t; precision is made
monotone and sampled at 101 recall points; AP is averaged over classes with
ground truth, and mAP over t in 0.50:0.05:0.95.  (No crowd / area ranges.)
"""
from __future__ import annotations

from typing import Dict, List, Sequence

import torch

from .ops import box_iou


def _ap_at(dets, gts, cls: int, t: float) -> float | None:
    recs = []
    n_gt = 0
    for img, (d, g) in enumerate(zip(dets, gts)):
        gm = g["labels"] == cls
        n_gt += int(gm.sum())
        dm = d["labels"] == cls
        for s, bi in zip(d["scores"][dm].tolist(), dm.nonzero().squeeze(1).tolist()):
            recs.append((s, img, bi))
    if n_gt == 0:
        return None
    if not recs:
        return 0.0
    recs.sort(key=lambda r: -r[0])
    used = {}
    tp = []
    for s, img, bi in recs:
        g = gts[img]
        gm = (g["labels"] == cls).nonzero().squeeze(1)
        if gm.numel() == 0:
            tp.append(0)
            continue
        iou = box_iou(dets[img]["boxes"][bi:bi + 1].float(), g["boxes"][gm].float())[0]
        taken = used.setdefault(img, set())
        best, bj = -1.0, -1
        for j, v in enumerate(iou.tolist()):
            if v >= t and int(gm[j]) not in taken and v > best:
                best, bj = v, int(gm[j])
        if bj >= 0:
            taken.add(bj)
            tp.append(1)
        else:
            tp.append(0)
    tp_t = torch.tensor(tp, dtype=torch.float64)
    ctp = tp_t.cumsum(0)
    cfp = (1 - tp_t).cumsum(0)
    rec = ctp / n_gt
    prec = ctp / (ctp + cfp)
    for i in range(len(prec) - 2, -1, -1):  # monotone envelope
        prec[i] = max(prec[i], prec[i + 1])
    grid = torch.linspace(0, 1, 101, dtype=torch.float64)
    idx = torch.searchsorted(rec, grid, right=False)
    sampled = torch.where(idx < len(prec), prec[idx.clamp(max=len(prec) - 1)],
                          torch.zeros_like(grid))
    return float(sampled.mean())


def evaluate_detections(detections: Sequence[Dict[str, torch.Tensor]],
                        ground_truth: Sequence[Dict[str, torch.Tensor]],
                        num_classes: int) -> Dict[str, float]:
    """``detections``: per image {boxes, scores, labels}; ``ground_truth``: per image
    {boxes, labels}.  Returns mAP (0.50:0.95), AP50, AP75."""
    dets = [{k: v.detach().cpu() for k, v in d.items() if torch.is_tensor(v)} for d in detections]
    gts = [{k: v.detach().cpu() for k, v in g.items() if torch.is_tensor(v)} for g in ground_truth]
    per_t: List[float] = []
    ap50 = ap75 = 0.0
    for t in [0.5 + 0.05 * i for i in range(10)]:
        aps = [a for a in (_ap_at(dets, gts, c, t) for c in range(num_classes)) if a is not None]
        m = sum(aps) / len(aps) if aps else 0.0
        per_t.append(m)
        if abs(t - 0.5) < 1e-9:
            ap50 = m
        if abs(t - 0.75) < 1e-9:
            ap75 = m
    return {"mAP": sum(per_t) / len(per_t), "AP50": ap50, "AP75": ap75}
