"""Diagnostics of a trained sensor-fusion classifier.

Counterpart of complexity/generative/sensor_fusion/diagnostics.py:62-360:

* ``hash_route_diagnostics``: for every TR-Hash FFN of the model, how many
  (route, slot) entries of its fixed route table land on each expert -- the
  load balance that the hash routing promises, checked on the checkpoint;
* ``evaluate_sensor_mode``: accuracy / macro-F1 / loss with all streams, or
  with one stream alone (samples without it are skipped, the others are
  masked out), overall and per subject;
* ``evaluate_late_fusion_sweep``: re-mixes the fused head and the
  per-stream heads on held-out data without touching parameters, over a
  grid of late-fusion weights, gate temperatures and per-stream boosts, and
  reports the best setting.

Batches are ``(inputs, masks, labels[, subject_ids])`` as produced by
``collate_sensors_masked`` (plus subject ids).
"""
from __future__ import annotations

import itertools
from typing import Dict, Iterable, Mapping, Optional

import torch
import torch.nn.functional as F

from .sensor_fusion import SENSOR_MODALITIES
from .sensor_training import classification_metrics_from_confusion


def hash_route_diagnostics(model) -> Dict[str, Dict]:
    from ..tr_hash.engine import TRHashEngine

    out = {}
    for name, mod in model.named_modules():
        if not isinstance(mod, TRHashEngine):
            continue
        table = mod.route_table.detach().long().cpu()
        E = int(mod.config.num_experts)
        counts = torch.bincount(table.flatten(), minlength=E)
        k_dim = 0 if table.shape[0] == mod.config.top_k else 1
        out[name] = {"routes": int(table.shape[1 - k_dim]), "top_k": int(table.shape[k_dim]),
                     "expert_assignments": counts.tolist(),
                     "expert_shares": (counts.double() / max(1, int(counts.sum()))).tolist(),
                     "max_over_mean": float(counts.max() / counts.double().mean().clamp_min(1e-12))}
    return {"layers": out}


def _unpack(batch, device):
    inputs, masks, labels = batch[:3]
    subj = batch[3] if len(batch) > 3 else None
    mv = lambda d: {k: v.to(device) for k, v in d.items()}  # noqa: E731
    return mv(inputs), mv(masks), labels.to(device), subj


def _confusion(labels, pred, C):
    return torch.bincount(labels * C + pred, minlength=C * C).view(C, C).cpu()


@torch.no_grad()
def evaluate_sensor_mode(model, batches: Iterable, device, modality: Optional[str] = None
                         ) -> Dict:
    if modality is not None and modality not in SENSOR_MODALITIES:
        raise ValueError(f"unknown modality {modality!r}")
    model.eval()
    C = model.config.num_classes
    conf = torch.zeros(C, C, dtype=torch.long)
    per_subject: Dict[int, torch.Tensor] = {}
    loss_sum, n = 0.0, 0
    for batch in batches:
        inputs, masks, labels, subj = _unpack(batch, device)
        if modality is not None:
            if modality not in inputs:
                continue
            keep = masks[modality].bool()
            if not bool(keep.any()):
                continue
            inputs = {modality: inputs[modality][keep]}
            masks = {modality: masks[modality][keep]}
            labels = labels[keep]
            subj = subj[keep.cpu()] if subj is not None else None
        out = model(inputs, labels=labels, masks=masks)
        pred = out["logits"].argmax(-1)
        conf += _confusion(labels, pred, C)
        if subj is not None:
            for s in subj.unique().tolist():
                sel = (subj == s).to(labels.device)
                per_subject.setdefault(int(s), torch.zeros(C, C, dtype=torch.long))
                per_subject[int(s)] += _confusion(labels[sel], pred[sel], C)
        loss_sum += float(out["loss"]) * labels.numel()
        n += labels.numel()
    m = classification_metrics_from_confusion(conf)
    m.update(validation_loss=loss_sum / max(1, n), mode=modality or "all", examples=n,
             by_subject={str(s): classification_metrics_from_confusion(c)
                         for s, c in sorted(per_subject.items())})
    return m


@torch.no_grad()
def evaluate_late_fusion_sweep(model, batches: Iterable, device,
                               late_weights=(0.0, 0.1, 0.25, 0.5, 1.0, 2.0),
                               gate_temperatures=(0.25, 0.5, 1.0, 2.0, 4.0),
                               stream_boosts: Optional[Mapping[str, Iterable[float]]] = None
                               ) -> Dict:
    """Best (late weight w, gate temperature T, per-stream boosts) by macro-F1.

    The re-mixed logits are ``(fused + w * per_stream) / (1 + w)``, where
    ``per_stream`` averages the stream heads with weights
    ``softmax(log(gate weight * boost) / T)`` over the streams present."""
    lw = tuple(float(v) for v in late_weights)
    ts = tuple(float(v) for v in gate_temperatures)
    boosts = {m: tuple(float(b) for b in bs) for m, bs in (stream_boosts or
                                                            {"skeleton": (1.0, 2.0, 4.0)}).items()}
    if not lw or min(lw) < 0:
        raise ValueError("late-fusion weights must be non-empty and non-negative")
    if not ts or min(ts) <= 0:
        raise ValueError("gate temperatures must be positive")
    if any(min(b) <= 0 for b in boosts.values()):
        raise ValueError("stream boosts must be positive")
    model.eval()
    L, FU, ML, MW, MM = [], [], [], [], []
    for batch in batches:
        inputs, masks, labels, _ = _unpack(batch, device)
        out = model(inputs, masks=masks)
        L.append(labels.cpu())
        FU.append(out["fused_logits"].float().cpu())
        ML.append(out["modality_logits"].float().cpu())
        MW.append(out["modality_weights"].float().cpu())
        MM.append(out["modality_mask"].cpu())
    labels, fused = torch.cat(L), torch.cat(FU)
    mlog, mw, mm = torch.cat(ML), torch.cat(MW), torch.cat(MM)
    C = model.config.num_classes
    idx = {m: i for i, m in enumerate(SENSOR_MODALITIES)}
    names = sorted(boosts)
    results = []
    for w, T, combo in itertools.product(lw, ts, itertools.product(*(boosts[m] for m in names))):
        scale = torch.ones(len(SENSOR_MODALITIES))
        for m, b in zip(names, combo):
            scale[idx[m]] = b
        logit = (mw.clamp_min(1e-12) * scale).log() / T
        g = logit.masked_fill(~mm, float("-inf")).softmax(1)
        per = (mlog * g[..., None]).sum(1)
        logits = (fused + w * per) / (1.0 + w)
        met = classification_metrics_from_confusion(_confusion(labels, logits.argmax(-1), C))
        met["loss"] = float(F.cross_entropy(logits, labels))
        results.append({"late_weight": w, "gate_temperature": T,
                        "boosts": dict(zip(names, combo)), **met})
    best = max(results, key=lambda r: (r["macro_f1"], r["accuracy"], -r["loss"]))
    return {"best": best, "results": results, "examples": int(labels.numel())}


__all__ = ["evaluate_late_fusion_sweep", "evaluate_sensor_mode", "hash_route_diagnostics"]
