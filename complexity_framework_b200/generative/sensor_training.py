"""Training of the TR-Hash sensor-fusion classifier.

Counterpart of complexity/generative/sensor_fusion/training.py:297-1646.
  * Augmentation schedule: full strength through the noisy phase, then a
    linear anneal to zero across the final ``clean_finetune_epochs``; the
    temporal-jitter switch is drawn per epoch with that probability.
  * Batch augmentation: per-sample modality dropout (never hides every
    stream of a sample: the first available one is kept), visual gain/offset
    jitter, additive sensor noise, mixup (Beta(alpha, alpha) weight; the
    mixed sample keeps the union of both samples' streams).
  * Imbalance handling: class weights (inverse or inverse-sqrt frequency,
    mean one over present classes), sampling weights, per-sample loss weights
    from action x subject (x completeness) frequencies, rescaled to mean one
    within optional hard bounds (the scale found by bisection).
  * Objectives: sample-weighted cross-entropy, auxiliary per-modality
    cross-entropy over the available streams, a gate-calibration loss (the
    learned modality gate is pulled toward a softmax of each stream's
    detached per-example quality, with a small uniform floor), and a
    supervised contrastive loss whose candidates are the features of every
    rank (autograd-aware all-gather).
  * Evaluation: accuracy and macro-F1 from the confusion matrix.
  * ``train_sensor_fusion``: epochs over a manifest with all of the above,
    AdamW + warmup cosine, EMA-free, best-by-macro-F1 checkpoint.
"""
from __future__ import annotations

import json
import math
import random
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .sensor_fusion import SENSOR_MODALITIES, SensorRecord, TRHashSensorFusionClassifier


# -------------------------------------------------------------- schedules
def augmentation_scale(epoch: int, *, total_epochs: int, clean_finetune_epochs: int) -> float:
    if clean_finetune_epochs <= 0 or total_epochs <= 0:
        return 1.0
    start = max(total_epochs - clean_finetune_epochs, 0)
    if epoch < start:
        return 1.0
    return max(0.0, 1.0 - min((epoch - start) / max(clean_finetune_epochs, 1), 1.0))


def clean_finetune_anneal_start(*, total_epochs: int, clean_finetune_epochs: int) -> int:
    if clean_finetune_epochs <= 0 or total_epochs <= 0:
        return total_epochs
    return max(total_epochs - clean_finetune_epochs, 0)


def resolve_epoch_training_augmentation(*, base_enabled: bool, aug_scale: float, seed: int,
                                        epoch: int) -> bool:
    return base_enabled and random.Random(seed + epoch).random() < aug_scale


# ----------------------------------------------------------- augmentation
def apply_modality_dropout(masks: Mapping[str, torch.Tensor],
                           probability: float) -> Dict[str, torch.Tensor]:
    if not 0.0 <= probability < 1.0:
        raise ValueError("modality_dropout must be in [0, 1)")
    names = tuple(masks)
    out = {n: masks[n].clone() for n in names}
    if probability == 0.0 or not names:
        return out
    have = torch.stack([out[n] for n in names], 1).bool()
    kept = have & (torch.rand(have.shape, device=have.device) >= probability)
    none = ~kept.any(1)
    if bool(none.any()):
        first = have.to(torch.int64).argmax(1)
        kept[none, first[none]] = True
    return {n: kept[:, i] for i, n in enumerate(names)}


def augment_sensor_inputs(inputs: Mapping[str, torch.Tensor], *, visual_jitter: float,
                          sensor_noise: float) -> Dict[str, torch.Tensor]:
    """Clips ([B, T, C, H, W]) get a per-sample gain in 1 +- j and offset in
    +- j/2 (clamped to [-1, 1]); sequences get Gaussian noise of std ``sensor_noise``."""
    if visual_jitter < 0.0 or sensor_noise < 0.0:
        raise ValueError("augmentation strengths must be non-negative")
    out = {}
    for n, v in inputs.items():
        if v.ndim == 5 and visual_jitter > 0.0:
            shape = (v.shape[0], 1, 1, 1, 1)
            gain = 1.0 + (2 * torch.rand(shape, device=v.device) - 1) * visual_jitter
            off = (2 * torch.rand(shape, device=v.device) - 1) * (0.5 * visual_jitter)
            out[n] = (v * gain + off).clamp(-1.0, 1.0)
        elif v.ndim in (3, 4) and sensor_noise > 0.0:
            out[n] = v + sensor_noise * torch.randn_like(v)
        else:
            out[n] = v
    return out


def mixup_sensor_batch(inputs, masks, labels: torch.Tensor, alpha: float):
    """-> (inputs, masks, partner labels, weight, permutation)."""
    if alpha < 0.0:
        raise ValueError("mixup_alpha must be non-negative")
    if alpha == 0.0 or labels.numel() < 2:
        return dict(inputs), dict(masks), labels, 1.0, torch.arange(labels.numel(),
                                                                    device=labels.device)
    lam = float(torch.distributions.Beta(alpha, alpha).sample())
    perm = torch.randperm(labels.numel(), device=labels.device)
    mixed = {n: lam * v + (1 - lam) * v[perm] for n, v in inputs.items()}
    mm = {n: v | v[perm] for n, v in masks.items()}
    return mixed, mm, labels[perm], lam, perm


# ---------------------------------------------------------- weighting
def _labels(records: Sequence[SensorRecord]) -> torch.Tensor:
    return torch.tensor([r.label for r in records], dtype=torch.long)


def build_class_weights(records, *, num_classes: int, mode: str, device=None):
    counts = torch.bincount(_labels(records), minlength=num_classes)
    present = counts > 0
    if not bool(present.any()):
        raise ValueError("cannot build class weights from an empty training split")
    if mode == "none":
        return None, counts
    w = torch.zeros(num_classes)
    if mode == "inverse-sqrt":
        w[present] = counts[present].float().rsqrt()
    elif mode == "inverse":
        w[present] = counts[present].float().reciprocal()
    else:
        raise ValueError(f"unsupported class balance mode: {mode}")
    w[present] /= w[present].mean()
    return (w.to(device) if device is not None else w), counts


def build_sampling_weights(records, *, num_classes: int, mode: str) -> torch.Tensor:
    lab = _labels(records)
    if mode == "none":
        return torch.ones(len(lab), dtype=torch.float64)
    counts = torch.bincount(lab, minlength=num_classes).double()
    if mode == "inverse-sqrt":
        cw = counts.clamp_min(1).rsqrt()
    elif mode == "inverse":
        cw = counts.clamp_min(1).reciprocal()
    else:
        raise ValueError(f"unsupported class sampling mode: {mode}")
    return cw[lab]


def normalize_bounded_weights(w: torch.Tensor, *, minimum: float, maximum: float) -> torch.Tensor:
    """Mean-one weights; with bounds, the scale s for which clamp(w s, lo, hi)
    has mean one, found by bisection."""
    w = w / w.mean()
    if minimum <= 0.0 and maximum <= 0.0:
        return w
    lo_b, hi_b = max(0.0, float(minimum)), (float(maximum) if maximum > 0 else float("inf"))
    lo, hi = 0.0, 1.0
    while torch.clamp(w * hi, lo_b, hi_b).mean() < 1.0:
        hi *= 2.0
    for _ in range(64):
        mid = 0.5 * (lo + hi)
        if torch.clamp(w * mid, lo_b, hi_b).mean() < 1.0:
            lo = mid
        else:
            hi = mid
    return torch.clamp(w * hi, lo_b, hi_b)


def build_sample_loss_weights(records, *, num_classes: int, mode: str, minimum: float = 0.0,
                              maximum: float = 0.0) -> torch.Tensor:
    """inverse(-sqrt) of (action frequency x action-subject frequency), with
    the -3d mode also dividing by sqrt(action x completeness frequency)."""
    if mode == "none":
        return torch.ones(len(records), dtype=torch.float64)
    if mode not in ("inverse-sqrt-2d", "inverse-2d", "inverse-sqrt-3d"):
        raise ValueError(f"unsupported sample loss weighting mode: {mode}")
    lab = _labels(records)
    cf = torch.bincount(lab, minlength=num_classes).double()[lab]
    pairs: Dict[Tuple[int, int], int] = {}
    for r in records:
        pairs[(r.label, r.subject)] = pairs.get((r.label, r.subject), 0) + 1
    pf = torch.tensor([pairs[(r.label, r.subject)] for r in records], dtype=torch.float64)
    w = (cf.rsqrt() * pf.rsqrt()) if mode != "inverse-2d" else (cf.reciprocal() * pf.reciprocal())
    if mode == "inverse-sqrt-3d":
        keys = [(r.label, all(m in r.files for m in SENSOR_MODALITIES)) for r in records]
        kc: Dict = {}
        for k in keys:
            kc[k] = kc.get(k, 0) + 1
        w = w * torch.tensor([kc[k] for k in keys], dtype=torch.float64).rsqrt()
    return normalize_bounded_weights(w, minimum=minimum, maximum=maximum)


# ------------------------------------------------------------ objectives
def weighted_cross_entropy(logits, labels, sample_weights, *, class_weights=None,
                           label_smoothing: float = 0.0) -> torch.Tensor:
    loss = F.cross_entropy(logits.float(), labels, weight=class_weights,
                           label_smoothing=label_smoothing, reduction="none")
    w = sample_weights.to(loss.device, loss.dtype)
    return (loss * w).sum() / w.sum().clamp_min(1e-12)


def _available(mask) -> torch.Tensor:
    if isinstance(mask, Mapping):
        return torch.stack([mask[n] for n in SENSOR_MODALITIES], 1).bool()
    return mask.bool()


def auxiliary_modality_loss(modality_logits, modality_mask, labels, sample_weights=None, *,
                            class_weights=None, label_smoothing: float = 0.0) -> torch.Tensor:
    if modality_logits.ndim != 3:
        raise ValueError("modality_logits must have shape [batch, modality, class]")
    av = _available(modality_mask)
    if av.shape != modality_logits.shape[:2]:
        raise ValueError("modality mask and logits shapes do not match")
    lab = labels[:, None].expand_as(av)
    loss = F.cross_entropy(modality_logits[av].float(), lab[av], weight=class_weights,
                           label_smoothing=label_smoothing, reduction="none")
    if sample_weights is None:
        return loss.mean()
    w = sample_weights[:, None].expand_as(av)[av].to(loss.dtype)
    return (loss * w).sum() / w.sum().clamp_min(1e-12)


def modality_gate_calibration_loss(modality_logits, modality_weights, modality_mask, labels,
                                   sample_weights=None, *, quality_temperature: float = 1.0,
                                   target_smoothing: float = 0.1,
                                   label_smoothing: float = 0.0) -> torch.Tensor:
    if modality_logits.ndim != 3:
        raise ValueError("modality_logits must have shape [batch, modality, class]")
    if modality_weights.shape not in (modality_logits.shape[:2], modality_logits.shape):
        raise ValueError("modality weights and logits shapes do not match")
    if labels.shape != (modality_logits.shape[0],):
        raise ValueError("labels must have shape [batch]")
    if quality_temperature <= 0.0:
        raise ValueError("gate quality temperature must be positive")
    if not 0.0 <= target_smoothing < 1.0:
        raise ValueError("gate target smoothing must be in [0, 1)")
    av = _available(modality_mask)
    if av.shape != modality_logits.shape[:2]:
        raise ValueError("modality mask and logits shapes do not match")
    if not bool(av.any(1).all()):
        raise ValueError("every example must expose at least one modality")
    B, M, C = modality_logits.shape
    q = F.cross_entropy(modality_logits.float().reshape(-1, C), labels[:, None].expand(B, M)
                        .reshape(-1), label_smoothing=label_smoothing,
                        reduction="none").view(B, M)
    tgt = (-q / quality_temperature).masked_fill(~av, float("-inf")).softmax(1).detach()
    if target_smoothing > 0.0:
        uni = av.float() / av.float().sum(1, keepdim=True)
        tgt = (1 - target_smoothing) * tgt + target_smoothing * uni
    w = modality_weights
    if w.ndim == 3:
        w = w.gather(2, labels[:, None, None].expand(-1, M, 1)).squeeze(-1)
    per = -(tgt * w.float().clamp_min(1e-8).log()).sum(1)
    if sample_weights is None:
        return per.mean()
    sw = sample_weights.to(per.device, per.dtype)
    return (per * sw).sum() / sw.sum().clamp_min(1e-12)


def supervised_contrastive_loss(features, labels, *, temperature: float = 0.1,
                                world: bool = False) -> torch.Tensor:
    """SupCon over this rank's anchors against every rank's features (``world``
    uses an autograd-aware all-gather, so each rank's gradient reaches the
    features it contributed)."""
    if features.ndim != 2:
        raise ValueError("contrastive features must have shape [batch, hidden]")
    if labels.shape != (features.shape[0],):
        raise ValueError("contrastive labels must have shape [batch]")
    if temperature <= 0.0:
        raise ValueError("contrastive temperature must be positive")
    a = F.normalize(features.float(), dim=-1)
    cand, cand_lab, rank = a, labels, 0
    if world and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        import torch.distributed.nn.functional as dist_nn

        cand = torch.cat(tuple(dist_nn.all_gather(a)), 0)
        labs = [torch.empty_like(labels) for _ in range(dist.get_world_size())]
        dist.all_gather(labs, labels)
        cand_lab, rank = torch.cat(labs), dist.get_rank()
    logits = a @ cand.t() / temperature
    n = a.shape[0]
    not_self = torch.ones_like(logits, dtype=torch.bool)
    not_self[torch.arange(n), rank * n + torch.arange(n)] = False
    pos = labels[:, None].eq(cand_lab[None]) & not_self
    cnt = pos.sum(1)
    ok = cnt > 0
    if not bool(ok.any()):
        return cand.sum() * 0.0   # keeps every rank in the gather's backward
    logits = logits - logits.masked_fill(~not_self, float("-inf")).amax(1, keepdim=True).detach()
    logp = logits - (logits.exp() * not_self).sum(1, keepdim=True).clamp_min(1e-12).log()
    mean_pos = torch.where(pos, logp, torch.zeros_like(logp)).sum(1) / cnt.clamp_min(1)
    return -mean_pos[ok].mean()


# ------------------------------------------------------------- evaluation
def classification_metrics_from_confusion(conf: torch.Tensor) -> Dict[str, float]:
    conf = conf.double()
    tp = conf.diag()
    prec = tp / conf.sum(0).clamp_min(1e-12)
    rec = tp / conf.sum(1).clamp_min(1e-12)
    f1 = 2 * prec * rec / (prec + rec).clamp_min(1e-12)
    present = conf.sum(1) > 0
    return {"accuracy": float(tp.sum() / conf.sum().clamp_min(1)),
            "macro_f1": float(f1[present].mean()) if bool(present.any()) else 0.0,
            "macro_recall": float(rec[present].mean()) if bool(present.any()) else 0.0}


@torch.no_grad()
def evaluate(model, batches, num_classes: int, device) -> Dict[str, float]:
    model.eval()
    conf = torch.zeros(num_classes, num_classes, dtype=torch.long)
    for batch in batches:
        inputs, masks, labels = batch[:3]
        out = model({k: v.to(device) for k, v in inputs.items()},
                    masks={k: v.to(device) for k, v in masks.items()})
        pred = out["logits"].argmax(-1).cpu()
        conf += torch.bincount(labels * num_classes + pred,
                               minlength=num_classes ** 2).view(num_classes, num_classes)
    return classification_metrics_from_confusion(conf)


# ----------------------------------------------------------------- driver
@dataclass
class SensorTrainConfig:
    epochs: int = 30
    batch_size: int = 32
    learning_rate: float = 3e-4
    weight_decay: float = 0.05
    warmup_steps: int = 100
    min_lr_ratio: float = 0.05
    label_smoothing: float = 0.1
    class_balance: str = "inverse-sqrt"        # none | inverse | inverse-sqrt
    sample_weighting: str = "none"             # none | inverse-2d | inverse-sqrt-2d | -3d
    sample_weight_min: float = 0.0
    sample_weight_max: float = 0.0
    modality_dropout: float = 0.2
    visual_jitter: float = 0.1
    sensor_noise: float = 0.02
    mixup_alpha: float = 0.2
    clean_finetune_epochs: int = 0
    aux_modality_weight: float = 0.3
    gate_calibration_weight: float = 0.0
    contrastive_weight: float = 0.0
    contrastive_temperature: float = 0.1
    grad_clip: float = 1.0
    seed: int = 0
    output: str = "sensor_run"


def train_sensor_fusion(model: TRHashSensorFusionClassifier, train_batches, val_batches,
                        train_records: Sequence[SensorRecord], config: SensorTrainConfig,
                        device=None) -> Dict[str, Any]:
    """``train_batches`` / ``val_batches``: re-iterable (inputs, masks, labels)
    batches (``collate_sensors_masked``); the records give the label and
    subject statistics for the imbalance weights (in the batches' order is not
    needed: per-sample loss weights are looked up by label and subject)."""
    from .detection.schedule import cosine_schedule

    c = config
    dev = torch.device(device) if device is not None else next(model.parameters()).device
    nc = model.config.num_classes
    cw, _ = build_class_weights(train_records, num_classes=nc, mode=c.class_balance, device=dev)
    sw_all = build_sample_loss_weights(train_records, num_classes=nc, mode=c.sample_weighting,
                                       minimum=c.sample_weight_min, maximum=c.sample_weight_max)
    # per-(label, subject) lookup of the sample weights
    sw_map = {(r.label, r.subject): float(w) for r, w in zip(train_records, sw_all)}
    steps_per_epoch = sum(1 for _ in train_batches)
    total = steps_per_epoch * c.epochs
    opt = torch.optim.AdamW(model.parameters(), lr=c.learning_rate, weight_decay=c.weight_decay)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: cosine_schedule(
        s, warmup_steps=min(c.warmup_steps, total), total_steps=total, min_ratio=c.min_lr_ratio))
    torch.manual_seed(c.seed)
    out = Path(c.output)
    best, hist = -1.0, []
    t0 = time.time()
    for epoch in range(c.epochs):
        scale = augmentation_scale(epoch, total_epochs=c.epochs,
                                   clean_finetune_epochs=c.clean_finetune_epochs)
        model.train()
        tot, n = 0.0, 0
        for batch in train_batches:
            inputs, masks, labels = batch[:3]
            subjects = batch[3] if len(batch) > 3 else None
            inputs = {k: v.to(dev) for k, v in inputs.items()}
            masks = {k: v.to(dev) for k, v in masks.items()}
            labels = labels.to(dev)
            masks = apply_modality_dropout(masks, c.modality_dropout * scale)
            inputs = augment_sensor_inputs(inputs, visual_jitter=c.visual_jitter * scale,
                                           sensor_noise=c.sensor_noise * scale)
            inputs, masks, partner, lam, perm = mixup_sensor_batch(inputs, masks, labels,
                                                                   c.mixup_alpha * scale)
            if subjects is not None:
                sw = torch.tensor([sw_map.get((int(l), int(s)), 1.0)
                                   for l, s in zip(labels.tolist(), subjects.tolist())],
                                  device=dev)
            else:
                sw = torch.ones(len(labels), device=dev)
            o = model(inputs, masks=masks)
            loss = lam * weighted_cross_entropy(o["logits"], labels, sw, class_weights=cw,
                                                label_smoothing=c.label_smoothing)
            if lam < 1.0:
                loss = loss + (1 - lam) * weighted_cross_entropy(
                    o["logits"], partner, sw[perm], class_weights=cw,
                    label_smoothing=c.label_smoothing)
            mm = o["modality_mask"]
            if c.aux_modality_weight > 0:
                loss = loss + c.aux_modality_weight * auxiliary_modality_loss(
                    o["modality_logits"], mm, labels, sw, class_weights=cw,
                    label_smoothing=c.label_smoothing)
            if c.gate_calibration_weight > 0 and model.config.modality_gate:
                loss = loss + c.gate_calibration_weight * modality_gate_calibration_loss(
                    o["modality_logits"], o["modality_weights"], mm, labels, sw)
            if c.contrastive_weight > 0:
                loss = loss + c.contrastive_weight * supervised_contrastive_loss(
                    o["features"], labels, temperature=c.contrastive_temperature, world=True)
            opt.zero_grad(set_to_none=True)
            loss.backward()
            torch.nn.utils.clip_grad_norm_(model.parameters(), c.grad_clip)
            opt.step()
            sched.step()
            tot, n = tot + float(loss.detach()), n + 1
        metrics = evaluate(model, val_batches, nc, dev)
        rec = {"epoch": epoch + 1, "train_loss": tot / max(n, 1), "aug_scale": scale,
               "seconds": time.time() - t0, **metrics}
        hist.append(rec)
        if metrics["macro_f1"] > best:
            best = metrics["macro_f1"]
            out.mkdir(parents=True, exist_ok=True)
            torch.save(model.state_dict(), out / "best_model.pt")
            (out / "best.json").write_text(json.dumps(
                {"config": model.config.to_dict(), "train": asdict(c), **rec}, indent=2,
                default=str))
    return {"best_macro_f1": best, "history": hist}
