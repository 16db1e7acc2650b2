"""Detector training run: epochs, accumulation, Mosaic closing, EMA, validation,
best-checkpoint selection and exact resume, one process per GPU.

    python -m complexity_framework_b200.generative.detection.train \
        --dataset synthetic --epochs 20 --batch-size 16 --output runs/det
    torchrun --nproc-per-node 8 -m complexity_framework_b200.generative.detection.train \
        --dataset coco --train-annotations .../instances_train2017.json --train-images ... \
        --val-annotations ... --val-images ... --image-size 640 --epochs 300

Counterpart of complexity/generative/detection/training.py:1474-2600 (the
``main`` loop).  Per epoch: the Mosaic probability is on until
``close_mosaic_epochs`` before the end; microbatches are grouped for gradient
accumulation (DDP synchronises only on group boundaries; a short final group
is averaged over its own size); each optimizer step clips gradients, steps a
per-step cosine schedule with warmup and updates the EMA.  After each epoch
``last/`` holds the EMA weights and the exact training state; on validation
epochs the EMA model is scored with the COCO-style accumulator (each rank
scores its shard, states are merged on rank 0) and ``best/`` follows the
selection score.  ``--resume`` continues from ``last/`` at the exact next
step (same run shape and options required).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import shutil
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Dict, List, Optional

import torch
from torch.utils.data import DataLoader

from .augmentations import AugmentedDataset, DetectionAugment
from .checkpointing import load_training_state, save_training_state
from .config import TRHashDetectorConfig
from .data import CocoDetectionDataset, SyntheticShapesDataset, YoloDetectionDataset, collate_detection
from .distributed import DistributedContext
from .ema import ModelEMA
from .exporting import save_detector_checkpoint
from .metrics import DetectionMetricsAccumulator
from .model import TRHashObjectDetector
from .schedule import (accumulation_group, cosine_schedule, detector_step_schedule,
                       mosaic_is_active_epoch, normalized_weight_decay,
                       optimizer_step_schedule, resolve_accumulation_steps, resolve_warmup_steps,
                       should_validate_epoch, validation_selection_score)

# options that must not change across an exact resume
RESUME_KEYS = ("dataset", "image_size", "num_classes", "batch_size", "nominal_batch_size",
               "accumulation_steps", "learning_rate", "min_lr_ratio", "weight_decay",
               "mosaic_probability", "close_mosaic_epochs", "packed_epochs",
               "mosaic_packed_epoch", "seed", "backbone")


@dataclass
class DetectorRunConfig:
    dataset: str = "synthetic"                 # synthetic | coco | yolo
    train_annotations: Optional[str] = None    # coco: instances json; yolo: list file
    train_images: Optional[str] = None
    val_annotations: Optional[str] = None
    val_images: Optional[str] = None
    synthetic_train: int = 256
    synthetic_val: int = 64
    image_size: int = 128
    num_classes: int = 2
    backbone: str = "plain"
    model_overrides: Dict = field(default_factory=dict)
    epochs: int = 10
    batch_size: int = 16
    nominal_batch_size: int = 64
    accumulation_steps: int = 0
    learning_rate: float = 1e-3
    min_lr_ratio: float = 0.05
    weight_decay: float = 0.05
    warmup_steps: int = 100
    warmup_epochs: Optional[float] = None
    grad_clip: float = 10.0
    ema_decay: float = 0.9998
    ema_tau: float = 200.0
    mosaic_probability: float = 0.5
    close_mosaic_epochs: int = 2
    packed_epochs: int = 1
    mosaic_packed_epoch: bool = False
    eval_every: int = 1
    confidence_threshold: float = 0.25
    amp_bf16: bool = True
    num_workers: int = 0
    seed: int = 0
    output: str = "detector_run"
    resume: bool = False
    device: Optional[str] = None


def _datasets(c: DetectorRunConfig):
    if c.dataset == "synthetic":
        return (SyntheticShapesDataset(c.synthetic_train, c.image_size, num_classes=c.num_classes,
                                       seed=c.seed),
                SyntheticShapesDataset(c.synthetic_val, c.image_size, num_classes=c.num_classes,
                                       seed=c.seed + 1))
    if c.dataset == "coco":
        return (CocoDetectionDataset(c.train_annotations, c.train_images, c.image_size),
                CocoDetectionDataset(c.val_annotations, c.val_images, c.image_size))
    if c.dataset == "yolo":
        return (YoloDetectionDataset(c.train_annotations, c.image_size),
                YoloDetectionDataset(c.val_annotations, c.image_size))
    raise ValueError(f"unknown dataset {c.dataset!r}")


def _lr_lambda(warmup: int, total: int, min_ratio: float):
    return lambda s: cosine_schedule(s, warmup_steps=warmup, total_steps=total, min_ratio=min_ratio)


@torch.no_grad()
def evaluate(model: TRHashObjectDetector, dataset, ctx: DistributedContext, *, batch_size: int,
             confidence_threshold: float, num_classes: int) -> Dict[str, float]:
    """COCO-style metrics of ``model`` over ``dataset`` (every rank scores its
    shard; rank 0 merges and the result is broadcast)."""
    acc = DetectionMetricsAccumulator(num_classes)
    loader = DataLoader(dataset, batch_size=batch_size, sampler=ctx.eval_sampler(dataset),
                        shuffle=False, collate_fn=collate_detection)
    model.eval()
    for images, targets in loader:
        for p, t in zip(model.predict(images.to(ctx.device)), targets):
            acc.update_xyxy(p["boxes"], p["scores"], p["labels"], t["boxes"], t["labels"])
    states = ctx.all_gather_objects(acc.state_dict())
    result = None
    if ctx.is_main:
        merged = DetectionMetricsAccumulator(num_classes)
        for st in states:
            merged.merge_state_dict(st)
        result = merged.compute(confidence_threshold)
    return ctx.broadcast_object(result)


def train_detector(c: DetectorRunConfig) -> Dict:
    dev = torch.device(c.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    ctx = DistributedContext.initialize(dev)
    dev = ctx.device
    torch.manual_seed(c.seed + ctx.rank)
    out = Path(c.output)
    train_ds, val_ds = _datasets(c)
    mcfg = TRHashDetectorConfig(image_size=c.image_size, num_classes=c.num_classes,
                                backbone=c.backbone, **c.model_overrides)
    torch.manual_seed(c.seed)  # identical initial weights on every rank
    model = TRHashObjectDetector(mcfg).to(dev)
    aug = DetectionAugment(train_ds, p_mosaic=c.mosaic_probability, seed=c.seed + 7 * ctx.rank)
    train_aug = AugmentedDataset(train_ds, aug)
    sampler = ctx.train_sampler(train_aug, c.seed)
    loader = DataLoader(train_aug, batch_size=c.batch_size, sampler=sampler,
                        shuffle=sampler is None, collate_fn=collate_detection,
                        num_workers=c.num_workers, drop_last=False)
    accum = resolve_accumulation_steps(per_device_batch_size=c.batch_size,
                                       world_size=ctx.world_size,
                                       nominal_batch_size=c.nominal_batch_size,
                                       requested_steps=c.accumulation_steps)
    micro = detector_step_schedule(len(loader), total_epochs=c.epochs,
                                   mosaic_probability=c.mosaic_probability,
                                   close_mosaic_epochs=c.close_mosaic_epochs,
                                   mosaic_packed_epoch=c.mosaic_packed_epoch,
                                   packed_epochs=c.packed_epochs)
    opt_steps = optimizer_step_schedule(micro, accum)
    total = sum(opt_steps)
    unpacked = sum(optimizer_step_schedule([len(loader)] * c.epochs, accum))
    warmup = resolve_warmup_steps(requested_steps=c.warmup_steps, warmup_epochs=c.warmup_epochs,
                                  steps_in_first_epoch=opt_steps[0], total_steps=total,
                                  unpacked_total_steps=unpacked)
    wd = normalized_weight_decay(c.weight_decay, global_batch_size=c.batch_size * ctx.world_size,
                                 accumulation_steps=accum, nominal_batch_size=c.nominal_batch_size)
    decay, no_decay = [], []
    for n, p in model.named_parameters():
        (no_decay if p.ndim < 2 or "norm" in n else decay).append(p)
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": wd},
                             {"params": no_decay, "weight_decay": 0.0}],
                            lr=c.learning_rate, betas=(0.9, 0.999))
    sched = torch.optim.lr_scheduler.LambdaLR(opt, _lr_lambda(warmup, total, c.min_lr_ratio))
    ema = ModelEMA(model, c.ema_decay, c.ema_tau)
    wrapped = ctx.wrap(model)
    options = {k: (v if not isinstance(v, tuple) else list(v)) for k, v in asdict(c).items()
               if k in RESUME_KEYS}
    step, start_epoch, skip, best = 0, 0, 0, -1.0
    run_losses: Dict[str, float] = {}
    run_steps = 0
    if c.resume and (out / "last").is_dir():
        sd = torch.load(out / "last" / "train_model.pt", map_location="cpu")
        model.load_state_dict(sd)
        st = load_training_state(out / "last", opt, sched, total_epochs=c.epochs,
                                 steps_per_epoch=opt_steps[0], training_options=options, ema=ema,
                                 rank=ctx.rank, world_size=ctx.world_size, device=dev)
        step, start_epoch, skip, best = (st["step"], st["epoch"], st["batch_in_epoch"],
                                         st["best_map50"])
        run_losses, run_steps = dict(st["running_losses"]), st["running_loss_steps"]
        aug_states = st.get("extra", {}).get("augment_rng")
        if aug_states:
            aug.rng.setstate(aug_states[ctx.rank])
    history: List[Dict] = []
    amp = c.amp_bf16 and dev.type == "cuda"
    t0 = time.time()
    for epoch in range(start_epoch, c.epochs):
        aug.p_mosaic = c.mosaic_probability if mosaic_is_active_epoch(
            epoch, total_epochs=c.epochs, close_mosaic_epochs=c.close_mosaic_epochs,
            mosaic_probability=c.mosaic_probability) else 0.0
        if sampler is not None:
            sampler.set_epoch(epoch)
        n_micro = micro[epoch]
        it = iter(loader)
        model.train()
        for b in range(n_micro):
            try:
                images, targets = next(it)
            except StopIteration:  # packed epochs shorter than the loader never get here
                it = iter(loader)
                images, targets = next(it)
            if epoch == start_epoch and b < skip:
                continue  # batches already trained before the resumed checkpoint
            size, last = accumulation_group(b, epoch_batches=n_micro, accumulation_steps=accum)
            targets = [{k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in t.items()}
                       for t in targets]
            sync = contextlib.nullcontext() if (last or not ctx.enabled) else wrapped.no_sync()
            with sync:
                with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
                    outs = wrapped(images.to(dev, non_blocking=True), targets)
                (outs["loss"] / size).backward()
            for k, v in outs.items():
                if k.startswith("loss"):
                    run_losses[k] = run_losses.get(k, 0.0) + float(v.detach())
            run_steps += 1
            if last:
                torch.nn.utils.clip_grad_norm_(model.parameters(), c.grad_clip)
                opt.step()
                sched.step()
                opt.zero_grad(set_to_none=True)
                ema.update(model)
                step += 1
        skip = 0
        losses = ctx.mean_scalars({k: v / max(run_steps, 1) for k, v in run_losses.items()})
        rec = {"epoch": epoch + 1, "step": step, "lr": sched.get_last_lr()[0], **losses,
               "mosaic": aug.p_mosaic > 0, "seconds": time.time() - t0}
        run_losses, run_steps = {}, 0
        if should_validate_epoch(epoch, c.epochs, c.eval_every):
            metrics = evaluate(ema.ema, val_ds, ctx, batch_size=c.batch_size,
                               confidence_threshold=c.confidence_threshold,
                               num_classes=c.num_classes)
            key, score = validation_selection_score(metrics)
            rec.update({f"val_{k}": v for k, v in metrics.items()})
            if score > best and ctx.is_main:
                save_detector_checkpoint(model, str(out / "best"), ema)
                (out / "best" / "metrics.json").write_text(json.dumps(
                    {"epoch": epoch + 1, "step": step, key: score, **metrics}, indent=2))
            best = max(best, score)
        history.append(rec)
        rngs = ctx.gather_rng_states()
        aug_rngs = ctx.all_gather_objects(aug.rng.getstate())
        if ctx.is_main:
            save_detector_checkpoint(model, str(out / "last"), ema)
            torch.save(model.state_dict(), out / "last" / "train_model.pt")
            save_training_state(out / "last", opt, sched, epoch=epoch + 1, batch_in_epoch=0,
                                step=step, best_map50=best, running_losses={},
                                running_loss_steps=0, total_epochs=c.epochs,
                                steps_per_epoch=opt_steps[0], training_options=options, ema=ema,
                                distributed_rng_states=rngs, extra={"augment_rng": aug_rngs})
            with open(out / "history.jsonl", "a") as f:
                f.write(json.dumps(rec) + "\n")
        ctx.barrier()
    summary = {"epochs": c.epochs, "steps": step, "optimizer_steps_planned": total,
               "accumulation_steps": accum, "warmup_steps": warmup, "weight_decay": wd,
               "best_score": best, "history": history}
    if ctx.is_main:
        (out / "summary.json").write_text(json.dumps(summary, indent=2, default=float))
    return summary


def parse_args(argv=None) -> DetectorRunConfig:
    c = DetectorRunConfig()
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    for k, v in asdict(c).items():
        if isinstance(v, dict):
            ap.add_argument(f"--{k.replace('_', '-')}", type=json.loads, default=v,
                            help="JSON object")
        elif isinstance(v, bool):
            ap.add_argument(f"--{k.replace('_', '-')}", action="store_true", default=v)
        else:
            typ = type(v) if v is not None else (float if k == "warmup_epochs" else str)
            ap.add_argument(f"--{k.replace('_', '-')}", type=typ, default=v)
    return DetectorRunConfig(**vars(ap.parse_args(argv)))


def main(argv=None) -> Dict:
    return train_detector(parse_args(argv))


if __name__ == "__main__":
    main()
