"""Release evaluation of a detector: COCO-style accuracy plus inference
latency / throughput measured per batch.

Counterpart of complexity/scripts/evaluate_tr_hash_coco.py:34-200.  The
reference evaluates a one-to-many head decoded with NMS and, when the
checkpoint has one, an NMS-free one-to-one head, in that fixed order.  This
framework's detector decodes its one-to-many head with class-aware NMS; a
model exposing ``predict_nms_free`` offers the second branch.

Batches are timed on the device (CUDA events around forward + decode, after
``warmup`` untimed batches; the host clock on CPU).
"""
from __future__ import annotations

import statistics
import time
from typing import Dict, List, Sequence, Tuple

import torch

from .coco_evaluation import evaluate_detections

BRANCHES: Tuple[str, ...] = ("o2m-nms", "nms-free")


def percentile(values: Sequence[float], fraction: float) -> float:
    """Nearest-rank percentile (``fraction`` in [0, 1]); 0 for no values."""
    if not values:
        return 0.0
    s = sorted(values)
    return s[min(len(s) - 1, round((len(s) - 1) * fraction))]


def timing_summary(batch_seconds: Sequence[float], image_count: int) -> Dict[str, float]:
    ms = [t * 1e3 for t in batch_seconds]
    total = float(sum(batch_seconds))
    return {"mean_batch_ms": statistics.fmean(ms) if ms else 0.0,
            "p50_batch_ms": percentile(ms, 0.50), "p95_batch_ms": percentile(ms, 0.95),
            "p99_batch_ms": percentile(ms, 0.99),
            "images_per_second": image_count / total if total else 0.0,
            "measured_seconds": total}


def branches_to_run(requested: str, *, has_nms_free: bool) -> Tuple[str, ...]:
    branches = BRANCHES if requested == "both" else (requested,)
    if any(b not in BRANCHES for b in branches):
        raise ValueError(f"unknown branch {requested!r}; expected both or one of {BRANCHES}")
    if "nms-free" in branches and not has_nms_free:
        raise ValueError("the model has no NMS-free (one-to-one) branch")
    return branches


@torch.no_grad()
def evaluate_release(model, images: torch.Tensor, targets: Sequence[Dict[str, torch.Tensor]],
                     *, branch: str = "o2m-nms", batch_size: int = 16, warmup: int = 2,
                     score_threshold: float = 0.001) -> Dict[str, Dict]:
    """Per branch: ``{"metrics": mAP / AP50 / AP75, "timing": timing_summary}``
    over ``images`` [N, 3, H, W] and their ``targets`` ({boxes, labels})."""
    has_free = callable(getattr(model, "predict_nms_free", None))
    dev = next(model.parameters()).device
    model.eval()
    out: Dict[str, Dict] = {}
    for br in branches_to_run(branch, has_nms_free=has_free):
        run = (model.predict_nms_free if br == "nms-free"
               else lambda x: model.predict(x, score_threshold=score_threshold))
        batches = [images[i:i + batch_size] for i in range(0, len(images), batch_size)]
        for b in batches[:warmup]:
            run(b.to(dev))
        dets: List[Dict[str, torch.Tensor]] = []
        secs: List[float] = []
        for b in batches:
            x = b.to(dev)
            if dev.type == "cuda":
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                s.record()
                d = run(x)
                e.record()
                torch.cuda.synchronize()
                secs.append(s.elapsed_time(e) / 1e3)
            else:
                t0 = time.perf_counter()
                d = run(x)
                secs.append(time.perf_counter() - t0)
            dets.extend(d)
        out[br] = {"metrics": evaluate_detections(dets, targets, model.config.num_classes),
                   "timing": timing_summary(secs, len(images))}
    return out


__all__ = ["BRANCHES", "branches_to_run", "evaluate_release", "percentile", "timing_summary"]
