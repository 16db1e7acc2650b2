"""Training drivers of the text-to-image and instruction-editing models.

Counterparts of complexity/generative/image/training.py:41-463 and
image/edit_training.py:43-392: caption tokenisation with a validity mask,
rectified-flow loss steps with gradient accumulation and warmup-cosine
learning rate, an optional final SFT stage on a curated stream at a scaled
learning rate, EMA of the weights, pruned ``step_XXXXXXX`` checkpoints
(model, EMA, optimizer, scheduler; the training state written last) and
resume from the newest complete one.  Editing batches are
(source, target, instruction) and train with joint text / source dropout
(``image.sample_edit_condition_dropout``).
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch

from .detection.ema import ModelEMA
from .detection.schedule import cosine_schedule
from .vlm_training import latest_checkpoint, prune_checkpoints, stage_is_sft


def tokenize_captions(tokenizer, captions: Sequence[str], max_length: int,
                      device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(ids [B, L], mask [B, L] bool) right-padded; an empty caption becomes one
    pad token (still marked valid, so every row attends to something)."""
    pad = None
    if hasattr(tokenizer, "token_to_id"):
        pad = tokenizer.token_to_id("<pad>")
    if pad is None:
        pad = getattr(tokenizer, "pad_token_id", None)
    pad = 0 if pad is None else int(pad)
    enc = []
    for c in captions:
        e = tokenizer.encode(c)
        enc.append((list(e.ids) if hasattr(e, "ids") else list(e))[:max_length] or [pad])
    W = max(len(e) for e in enc)
    ids = torch.full((len(enc), W), pad, dtype=torch.long)
    mask = torch.zeros(len(enc), W, dtype=torch.bool)
    for i, e in enumerate(enc):
        ids[i, :len(e)] = torch.tensor(e)
        mask[i, :len(e)] = True
    if device is not None:
        ids, mask = ids.to(device, non_blocking=True), mask.to(device, non_blocking=True)
    return ids, mask


@dataclass
class ImageTrainConfig:
    max_steps: int = 1000
    sft_steps: int = 0
    sft_lr_scale: float = 0.2
    gradient_accumulation: int = 1
    max_text_length: int = 77
    learning_rate: float = 1e-4
    weight_decay: float = 0.0
    warmup_steps: int = 500
    min_lr_ratio: float = 0.1
    grad_clip: float = 1.0
    ema_decay: float = 0.9999
    ema_tau: float = 2000.0
    save_steps: int = 1000
    keep_checkpoints: int = 3
    log_steps: int = 20
    bf16: bool = True
    output: str = "image_run"
    resume: bool = False


def _cycle(src):
    while True:
        n = 0
        for b in src:
            n += 1
            yield b
        if n == 0:
            raise ValueError("empty batch source")


def _save(c: ImageTrainConfig, model, ema, opt, sched, step: int, stage: str) -> Path:
    d = Path(c.output) / f"step_{step:07d}"
    d.mkdir(parents=True, exist_ok=True)
    sd = {k: v for k, v in model.state_dict().items() if not k.startswith("codec.")}
    torch.save(sd, d / "model.pt")
    torch.save(ema.state_dict(), d / "ema.pt")
    (d / "meta.json").write_text(json.dumps({"step": step, "stage": stage}))
    torch.save({"step": step, "optimizer": opt.state_dict(), "scheduler": sched.state_dict()},
               d / ".training_state.tmp")
    (d / ".training_state.tmp").replace(d / "training_state.pt")
    prune_checkpoints(c.output, c.keep_checkpoints)
    return d


def train_image_model(model, tokenizer, batches: Iterable, config: ImageTrainConfig, *,
                      sft_batches: Optional[Iterable] = None, edit: bool = False) -> Dict:
    """Text-to-image batches are (images, captions); editing batches (``edit``)
    are (sources, targets, instructions).  Images are in [-1, 1]."""
    c = config
    dev = next(p for p in model.parameters() if p.requires_grad).device
    params = [p for n, p in model.named_parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=c.learning_rate, weight_decay=c.weight_decay)
    base = lambda s: cosine_schedule(s, warmup_steps=min(c.warmup_steps, c.max_steps),  # noqa: E731
                                     total_steps=c.max_steps, min_ratio=c.min_lr_ratio)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: base(s) * (
        c.sft_lr_scale if stage_is_sft(s, total_steps=c.max_steps, sft_steps=c.sft_steps)
        else 1.0))
    ema = ModelEMA(model, c.ema_decay, c.ema_tau)
    step = 0
    if c.resume:
        ck = latest_checkpoint(c.output)
        if ck is not None:
            model.load_state_dict(torch.load(ck / "model.pt", map_location="cpu"), strict=False)
            ema.load_state_dict(torch.load(ck / "ema.pt", map_location="cpu", weights_only=False))
            st = torch.load(ck / "training_state.pt", map_location="cpu", weights_only=False)
            opt.load_state_dict(st["optimizer"])
            sched.load_state_dict(st["scheduler"])
            step = st["step"]
    main, sft = _cycle(batches), (_cycle(sft_batches) if sft_batches is not None else None)
    amp = c.bf16 and dev.type == "cuda"
    log: List[Dict] = []
    while step < c.max_steps:
        in_sft = stage_is_sft(step, total_steps=c.max_steps, sft_steps=c.sft_steps)
        src = sft if (in_sft and sft is not None) else main
        model.train()
        opt.zero_grad(set_to_none=True)
        tot = 0.0
        for _ in range(c.gradient_accumulation):
            b = next(src)
            ids, _mask = tokenize_captions(tokenizer, b[-1], c.max_text_length, dev)
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
                if edit:
                    loss = model(source=b[0].to(dev), target=b[1].to(dev), text_ids=ids)["loss"]
                else:
                    loss = model(images=b[0].to(dev), text_ids=ids)["loss"]
            (loss / c.gradient_accumulation).backward()
            tot += float(loss.detach()) / c.gradient_accumulation
        torch.nn.utils.clip_grad_norm_(params, c.grad_clip)
        opt.step()
        sched.step()
        ema.update(model)
        step += 1
        stage = "sft" if in_sft else "pretrain"
        if step % c.log_steps == 0 or step == c.max_steps:
            log.append({"step": step, "loss": tot, "lr": sched.get_last_lr()[0], "stage": stage})
        if step % c.save_steps == 0 or step == c.max_steps:
            _save(c, model, ema, opt, sched, step, stage)
    return {"steps": step, "log": log, "ema": ema}
