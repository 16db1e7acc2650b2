"""Supervised pretraining of the TR-Hash vision tower (image classification).

    python -m complexity_framework_b200.generative.vision_pretraining \
        --train-dir data/imagenet/train --val-dir data/imagenet/val --epochs 90 --output runs/vit

Counterpart of complexity/generative/vision_language/pretraining.py:29-710:
the tower trains as ``TRHashVisionClassifier`` on an image-folder dataset
(one sub-directory per class; ``--synthetic`` uses generated images),
AdamW with a per-step cosine schedule and warmup, bf16 autocast, DDP through
the detection ``DistributedContext``, top-1 / top-5 validation each epoch,
``tower.pt`` (tower weights only, what the vision-language model loads) plus
the classifier and an exactly resumable training state after every epoch.
``ResumableBatchSampler`` skips already consumed batches by index, so a
mid-epoch resume decodes no image twice.
"""
from __future__ import annotations

import argparse
import json
import math
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Dict, Iterator, List, Optional

import torch
from torch.utils.data import DataLoader, Dataset, Sampler

from .detection.checkpointing import load_training_state, save_training_state
from .detection.distributed import DistributedContext
from .detection.schedule import cosine_schedule
from .towers import TRHashVisionClassifier, TRHashVisionTowerConfig


class ResumableBatchSampler(Sampler[List[int]]):
    """Epoch-seeded shuffled batches of this rank's stride of the dataset;
    ``skip`` drops the first batches (already trained) before any is loaded."""

    def __init__(self, n: int, batch_size: int, *, seed: int, rank: int = 0, world: int = 1,
                 drop_last: bool = True):
        self.n, self.bs, self.seed, self.rank, self.world = n, batch_size, seed, rank, world
        self.drop_last, self.epoch, self.skip = drop_last, 0, 0

    def set_epoch(self, epoch: int, skip: int = 0) -> None:
        self.epoch, self.skip = epoch, skip

    def _indices(self) -> List[int]:
        g = torch.Generator().manual_seed(self.seed + self.epoch)
        return torch.randperm(self.n, generator=g)[self.rank::self.world].tolist()

    def __iter__(self) -> Iterator[List[int]]:
        idx = self._indices()
        batches = [idx[i:i + self.bs] for i in range(0, len(idx), self.bs)]
        if self.drop_last and batches and len(batches[-1]) < self.bs:
            batches.pop()
        return iter(batches[self.skip:])

    def __len__(self) -> int:
        per = len(range(self.rank, self.n, self.world))
        full = per // self.bs if self.drop_last else -(-per // self.bs)
        return max(0, full - self.skip)


class SyntheticImageDataset(Dataset):
    """Class c = a bright square at a class-specific cell of a noisy image."""

    def __init__(self, length: int, image_size: int, num_classes: int, seed: int = 0):
        self.n, self.size, self.nc, self.seed = length, image_size, num_classes, seed

    def __len__(self) -> int:
        return self.n

    def __getitem__(self, i: int):
        g = torch.Generator().manual_seed(self.seed * 7919 + i)
        c = int(torch.randint(0, self.nc, (1,), generator=g))
        img = 0.2 * torch.rand(3, self.size, self.size, generator=g)
        k = math.ceil(math.sqrt(self.nc))
        cell = self.size // k
        y, x = (c // k) * cell, (c % k) * cell
        img[:, y:y + cell, x:x + cell] += 0.8
        return img.clamp(0, 1), c


def image_folder(root: str, image_size: int, train: bool):
    import torchvision.transforms as T
    from torchvision.datasets import ImageFolder

    tf = (T.Compose([T.RandomResizedCrop(image_size), T.RandomHorizontalFlip(), T.ToTensor()])
          if train else T.Compose([T.Resize(int(image_size * 1.14)), T.CenterCrop(image_size),
                                   T.ToTensor()]))
    return ImageFolder(root, transform=tf)


@dataclass
class VisionPretrainConfig:
    train_dir: Optional[str] = None
    val_dir: Optional[str] = None
    synthetic: bool = False
    synthetic_train: int = 512
    synthetic_val: int = 128
    num_classes: int = 10
    tower: Dict = field(default_factory=dict)     # TRHashVisionTowerConfig fields
    epochs: int = 10
    batch_size: int = 64
    learning_rate: float = 1e-3
    min_lr_ratio: float = 0.01
    weight_decay: float = 0.05
    warmup_steps: int = 500
    grad_clip: float = 1.0
    label_smoothing: float = 0.0
    bf16: bool = True
    num_workers: int = 4
    seed: int = 0
    output: str = "vision_pretrain"
    resume: bool = False
    device: Optional[str] = None


RESUME_KEYS = ("num_classes", "batch_size", "learning_rate", "min_lr_ratio", "weight_decay",
               "seed", "label_smoothing")


@torch.no_grad()
def validate(model, loader, ctx: DistributedContext) -> Dict[str, float]:
    model.eval()
    top1 = top5 = n = 0.0
    loss = 0.0
    for x, y in loader:
        x, y = x.to(ctx.device), y.to(ctx.device)
        logits = model(x)["logits"].float()
        loss += float(torch.nn.functional.cross_entropy(logits, y, reduction="sum"))
        k = min(5, logits.shape[1])
        pred = logits.topk(k, -1).indices
        top1 += float((pred[:, 0] == y).sum())
        top5 += float((pred == y[:, None]).any(1).sum())
        n += len(y)
    tot = ctx.all_gather_objects((top1, top5, loss, n))
    t1, t5, ls, nn_ = (sum(v[i] for v in tot) for i in range(4))
    return {"top1": t1 / max(nn_, 1), "top5": t5 / max(nn_, 1), "val_loss": ls / max(nn_, 1)}


def pretrain_vision_tower(c: VisionPretrainConfig) -> Dict:
    dev = torch.device(c.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    ctx = DistributedContext.initialize(dev)
    dev = ctx.device
    tcfg = TRHashVisionTowerConfig(**c.tower)
    if c.synthetic:
        train_ds = SyntheticImageDataset(c.synthetic_train, tcfg.image_size, c.num_classes, c.seed)
        val_ds = SyntheticImageDataset(c.synthetic_val, tcfg.image_size, c.num_classes, c.seed + 1)
    else:
        train_ds = image_folder(c.train_dir, tcfg.image_size, True)
        val_ds = image_folder(c.val_dir, tcfg.image_size, False)
    torch.manual_seed(c.seed)
    model = TRHashVisionClassifier(tcfg, c.num_classes).to(dev)
    bs = ResumableBatchSampler(len(train_ds), c.batch_size, seed=c.seed, rank=ctx.rank,
                               world=ctx.world_size)
    loader = DataLoader(train_ds, batch_sampler=bs, num_workers=c.num_workers,
                        pin_memory=dev.type == "cuda")
    vloader = DataLoader(val_ds, batch_size=c.batch_size, sampler=ctx.eval_sampler(val_ds),
                         num_workers=c.num_workers)
    steps_per_epoch = len(bs)
    total = steps_per_epoch * c.epochs
    decay = [p for n, p in model.named_parameters() if p.ndim >= 2]
    no_decay = [p for n, p in model.named_parameters() if p.ndim < 2]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": c.weight_decay},
                             {"params": no_decay, "weight_decay": 0.0}], lr=c.learning_rate)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: cosine_schedule(
        s, warmup_steps=min(c.warmup_steps, total), total_steps=total, min_ratio=c.min_lr_ratio))
    wrapped = ctx.wrap(model)
    options = {k: v for k, v in asdict(c).items() if k in RESUME_KEYS}
    out = Path(c.output)
    step, epoch0, skip, best = 0, 0, 0, -1.0
    if c.resume and (out / "last" / "training_state.pt").exists():
        model.load_state_dict(torch.load(out / "last" / "classifier.pt", map_location="cpu"))
        st = load_training_state(out / "last", opt, sched, total_epochs=c.epochs,
                                 steps_per_epoch=steps_per_epoch, training_options=options,
                                 rank=ctx.rank, world_size=ctx.world_size, device=dev)
        step, epoch0, skip, best = st["step"], st["epoch"], st["batch_in_epoch"], st["best_map50"]
    amp = c.bf16 and dev.type == "cuda"
    history = []
    t0 = time.time()
    for epoch in range(epoch0, c.epochs):
        bs.set_epoch(epoch, skip if epoch == epoch0 else 0)
        model.train()
        tot, cnt = 0.0, 0
        for x, y in loader:
            x, y = x.to(dev, non_blocking=True), y.to(dev, non_blocking=True)
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
                logits = wrapped(x)["logits"]
            loss = torch.nn.functional.cross_entropy(logits.float(), y,
                                                     label_smoothing=c.label_smoothing)
            opt.zero_grad(set_to_none=True)
            loss.backward()
            torch.nn.utils.clip_grad_norm_(model.parameters(), c.grad_clip)
            opt.step()
            sched.step()
            step += 1
            tot, cnt = tot + float(loss.detach()), cnt + 1
        metrics = validate(model, vloader, ctx)
        rec = {"epoch": epoch + 1, "step": step, "train_loss": tot / max(cnt, 1),
               "lr": sched.get_last_lr()[0], "seconds": time.time() - t0, **metrics}
        history.append(rec)
        rngs = ctx.gather_rng_states()
        if ctx.is_main:
            for d in (["last"] + (["best"] if metrics["top1"] > best else [])):
                (out / d).mkdir(parents=True, exist_ok=True)
                torch.save(model.tower.state_dict(), out / d / "tower.pt")
                torch.save(model.state_dict(), out / d / "classifier.pt")
                (out / d / "config.json").write_text(json.dumps(
                    {"tower": asdict(tcfg), "num_classes": c.num_classes, "metrics": rec},
                    indent=2))
            save_training_state(out / "last", opt, sched, epoch=epoch + 1, batch_in_epoch=0,
                                step=step, best_map50=max(best, metrics["top1"]),
                                running_losses={}, running_loss_steps=0, total_epochs=c.epochs,
                                steps_per_epoch=steps_per_epoch, training_options=options,
                                distributed_rng_states=rngs)
            with open(out / "history.jsonl", "a") as f:
                f.write(json.dumps(rec) + "\n")
        best = max(best, metrics["top1"])
        ctx.barrier()
    return {"steps": step, "best_top1": best, "history": history}


def main(argv=None) -> Dict:
    c = VisionPretrainConfig()
    ap = argparse.ArgumentParser(description="TR-Hash vision tower pretraining")
    for k, v in asdict(c).items():
        flag = f"--{k.replace('_', '-')}"
        if isinstance(v, bool):
            ap.add_argument(flag, action="store_true", default=v)
        elif isinstance(v, dict):
            ap.add_argument(flag, type=json.loads, default=v)
        else:
            ap.add_argument(flag, type=type(v) if v is not None else str, default=v)
    return pretrain_vision_tower(VisionPretrainConfig(**vars(ap.parse_args(argv))))


if __name__ == "__main__":
    main()
