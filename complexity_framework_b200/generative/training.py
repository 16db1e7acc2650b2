"""One training loop for every generative model here (counterpart:
complexity/generative/vision_language/pretraining.py + training.py,
image/training.py + edit_training.py and the audio trainer).  A model's
``forward(**batch)`` returns a dict with ``loss``; the loop adds AdamW (no
decay on norms / biases / 1-d parameters), warmup + cosine schedule, bf16
autocast on CUDA, gradient clipping, optional data parallel (one process per
GPU) and checkpoints of the trainable state."""
from __future__ import annotations

import math
import os
from dataclasses import asdict, dataclass
from typing import Dict, Iterable, Mapping, Optional

import torch


@dataclass
class GenerativeTrainingConfig:
    learning_rate: float = 3e-4
    weight_decay: float = 0.05
    warmup_steps: int = 100
    max_steps: int = 10000
    min_lr_ratio: float = 0.1
    grad_clip: float = 1.0
    amp_bf16: bool = True
    log_every: int = 50


class GenerativeTrainer:
    def __init__(self, model: torch.nn.Module, config: Optional[GenerativeTrainingConfig] = None):
        import torch.distributed as dist

        self.model = model
        self.config = c = config or GenerativeTrainingConfig()
        params = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
        decay = [p for n, p in params if p.ndim >= 2 and "norm" not in n]
        no_decay = [p for n, p in params if not (p.ndim >= 2 and "norm" not in n)]
        self.optimizer = torch.optim.AdamW([{"params": decay, "weight_decay": c.weight_decay},
                                            {"params": no_decay, "weight_decay": 0.0}],
                                           lr=c.learning_rate, betas=(0.9, 0.95))

        def mult(step):
            if step < c.warmup_steps:
                return (step + 1) / max(1, c.warmup_steps)
            t = min(1.0, (step - c.warmup_steps) / max(1, c.max_steps - c.warmup_steps))
            return c.min_lr_ratio + (1 - c.min_lr_ratio) * 0.5 * (1 + math.cos(math.pi * t))

        self.scheduler = torch.optim.lr_scheduler.LambdaLR(self.optimizer, mult)
        self.world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        self.wrapped = model
        if self.world > 1:
            dev = next(model.parameters()).device
            self.wrapped = torch.nn.parallel.DistributedDataParallel(
                model, device_ids=[dev.index] if dev.type == "cuda" else None,
                find_unused_parameters=True)
        self.step = 0

    def train_step(self, batch: Mapping) -> Dict[str, float]:
        dev = next(self.model.parameters()).device
        batch = {k: v.to(dev, non_blocking=True) if torch.is_tensor(v) else v
                 for k, v in batch.items()}
        self.model.train()
        amp = self.config.amp_bf16 and dev.type == "cuda"
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
            out = self.wrapped(**batch)
        self.optimizer.zero_grad(set_to_none=True)
        out["loss"].backward()
        if self.config.grad_clip > 0:
            torch.nn.utils.clip_grad_norm_(
                [p for p in self.model.parameters() if p.requires_grad], self.config.grad_clip)
        self.optimizer.step()
        self.scheduler.step()
        self.step += 1
        return {k: float(v.detach()) for k, v in out.items()
                if k.startswith("loss") and torch.is_tensor(v)}

    def train(self, batches: Iterable[Mapping], max_steps: Optional[int] = None, log=print):
        n = max_steps or self.config.max_steps
        last = {}
        for batch in batches:
            if self.step >= n:
                break
            last = self.train_step(batch)
            if log is not None and self.step % self.config.log_every == 0:
                log({"step": self.step, **last, "lr": self.scheduler.get_last_lr()[0]})
        return last

    def save(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        torch.save({"model": self.model.state_dict(), "optimizer": self.optimizer.state_dict(),
                    "scheduler": self.scheduler.state_dict(), "step": self.step,
                    "config": asdict(self.config)}, os.path.join(path, "trainer.pt"))

    def load(self, path: str) -> None:
        sd = torch.load(os.path.join(path, "trainer.pt"), map_location="cpu", weights_only=False)
        self.model.load_state_dict(sd["model"])
        self.optimizer.load_state_dict(sd["optimizer"])
        self.scheduler.load_state_dict(sd["scheduler"])
        self.step = sd["step"]
