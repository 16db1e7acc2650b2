"""Detector training loop (counterpart: complexity/generative/detection/trainer.py,
a 2,600-line loop with AMP, EMA, warmup, evaluation and checkpointing; this is
the same loop shape without the dataset-specific options).

AdamW with decoupled weight decay (no decay on norms / biases), linear warmup
then cosine decay, gradient clipping, EMA of the weights, periodic COCO-style
evaluation of the EMA model, bf16 autocast on CUDA.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Iterable, Optional

import torch

from .coco_evaluation import evaluate_detections
from .ema import ModelEMA
from .model import TRHashObjectDetector


@dataclass
class DetectorTrainingConfig:
    learning_rate: float = 1e-3
    weight_decay: float = 0.05
    warmup_steps: int = 100
    max_steps: int = 1000
    grad_clip: float = 10.0
    ema_decay: float = 0.9998
    ema_tau: float = 200.0
    amp_bf16: bool = True


class DetectorTrainer:
    def __init__(self, model: TRHashObjectDetector, config: Optional[DetectorTrainingConfig] = None):
        import torch.distributed as dist

        self.model = model
        # data parallel: one process per GPU; gradients are averaged by DDP
        self.world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        self.ddp = None
        if self.world > 1:
            dev = next(model.parameters()).device
            self.ddp = torch.nn.parallel.DistributedDataParallel(
                model, device_ids=[dev.index] if dev.type == "cuda" else None,
                find_unused_parameters=True)
        self.config = c = config or DetectorTrainingConfig()
        decay, no_decay = [], []
        for n, p in model.named_parameters():
            (no_decay if p.ndim < 2 or "norm" in n else decay).append(p)
        self.optimizer = torch.optim.AdamW([{"params": decay, "weight_decay": c.weight_decay},
                                            {"params": no_decay, "weight_decay": 0.0}],
                                           lr=c.learning_rate, betas=(0.9, 0.999))

        def lr_mult(step):
            if step < c.warmup_steps:
                return (step + 1) / max(1, c.warmup_steps)
            t = min(1.0, (step - c.warmup_steps) / max(1, c.max_steps - c.warmup_steps))
            return 0.05 + 0.95 * 0.5 * (1 + math.cos(math.pi * t))

        self.scheduler = torch.optim.lr_scheduler.LambdaLR(self.optimizer, lr_mult)
        self.ema = ModelEMA(model, c.ema_decay, c.ema_tau)
        self.step = 0

    def train_step(self, images: torch.Tensor, targets) -> Dict[str, float]:
        dev = next(self.model.parameters()).device
        self.model.train()
        images = images.to(dev, non_blocking=True)
        amp = self.config.amp_bf16 and dev.type == "cuda"
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
            out = (self.ddp or self.model)(images, targets)
        self.optimizer.zero_grad(set_to_none=True)
        out["loss"].backward()
        torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.config.grad_clip)
        self.optimizer.step()
        self.scheduler.step()
        self.ema.update(self.model)
        self.step += 1
        return {k: float(v.detach()) for k, v in out.items() if k.startswith("loss")}

    @torch.no_grad()
    def evaluate(self, loader: Iterable, use_ema: bool = True) -> Dict[str, float]:
        model = self.ema.ema if use_ema else self.model
        dev = next(model.parameters()).device
        dets, gts = [], []
        for images, targets in loader:
            dets += [{k: v.cpu() for k, v in d.items()} for d in model.predict(images.to(dev))]
            gts += [{k: v for k, v in t.items() if torch.is_tensor(v)} for t in targets]
        if self.world > 1:  # every rank evaluated its shard; score the union
            import torch.distributed as dist

            all_d, all_g = [None] * self.world, [None] * self.world
            dist.all_gather_object(all_d, dets)
            dist.all_gather_object(all_g, gts)
            dets = [d for part in all_d for d in part]
            gts = [g for part in all_g for g in part]
        return evaluate_detections(dets, gts, model.config.num_classes)
