"""Training of the TR-Hash image-text-to-text model: alignment, then a final
vision-only instruction (SFT) stage.

Counterpart of complexity/generative/vision_language/training.py:38-521.
  * ``tokenize_prompt_response``: prompt + response (+ EOS) per example, labels
    only on the response tokens, right padding;
  * ``stage_is_sft``: the last ``sft_steps`` optimizer steps form the SFT stage;
    entering it freezes the language decoder (``freeze_decoder_for_vision_only_sft``:
    the vision tower and resampler keep training, the decoder never does in
    this stage) and switches to the SFT batches;
  * checkpoints ``step_XXXXXXX/`` (model, optimizer, scheduler, step), the
    newest ``keep_checkpoints`` kept (``prune_checkpoints``), exact resume of
    the step counter and optimizer.
Data are (image, prompt, response) examples; ``PromptResponseTarDataset``
reads webdataset-style shards (``<key>.jpg|png``, ``<key>.txt`` response,
optional ``<key>.prompt``; a default prompt otherwise).
"""
from __future__ import annotations

import io
import json
import math
import shutil
import tarfile
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Dict, Iterable, Iterator, List, Optional, Sequence, Tuple

import torch

DEFAULT_PROMPT = "Describe the image."


def _encode(tok, text: str) -> List[int]:
    e = tok.encode(text)
    return list(e.ids) if hasattr(e, "ids") else list(e)


def _special(tok, name: str, attr: str) -> Optional[int]:
    if hasattr(tok, "token_to_id"):
        v = tok.token_to_id(name)
        if v is not None:
            return int(v)
    v = getattr(tok, attr, None)
    return None if v is None else int(v)


def tokenize_prompt_response(tokenizer, prompts: Sequence[str], responses: Sequence[str],
                             max_length: int, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(input_ids [B, T], labels [B, T]) with -100 on prompt and padding."""
    pad = _special(tokenizer, "<pad>", "pad_token_id")
    pad = 0 if pad is None else pad
    eos = _special(tokenizer, "</s>", "eos_token_id")
    seqs, plen = [], []
    for p, r in zip(prompts, responses):
        pi, ri = _encode(tokenizer, p), _encode(tokenizer, r)
        if eos is not None:
            ri = ri + [eos]
        s = (pi + ri)[:max_length] or [pad]
        seqs.append(s)
        plen.append(min(len(pi), len(s)))
    W = max(len(s) for s in seqs)
    ids = torch.full((len(seqs), W), pad, dtype=torch.long)
    lab = torch.full((len(seqs), W), -100, dtype=torch.long)
    for i, (s, n) in enumerate(zip(seqs, plen)):
        t = torch.tensor(s, dtype=torch.long)
        ids[i, :len(s)] = t
        lab[i, n:len(s)] = t[n:]
    if device is not None:
        ids, lab = ids.to(device, non_blocking=True), lab.to(device, non_blocking=True)
    return ids, lab


def stage_is_sft(step: int, *, total_steps: int, sft_steps: int) -> bool:
    return sft_steps > 0 and step >= total_steps - sft_steps


def freeze_decoder_for_vision_only_sft(model) -> Dict[str, int]:
    model.lm.decoder.requires_grad_(False)
    tr = sum(p.numel() for p in model.parameters() if p.requires_grad)
    tot = sum(p.numel() for p in model.parameters())
    return {"trainable": tr, "total": tot, "frozen": tot - tr}


def prune_checkpoints(output, keep_checkpoints: int) -> None:
    if keep_checkpoints <= 0:
        raise ValueError("keep_checkpoints must be positive")
    steps = sorted((p for p in Path(output).glob("step_*")
                    if p.is_dir() and p.name[5:].isdigit()), key=lambda p: int(p.name[5:]))
    for stale in steps[:-keep_checkpoints]:
        shutil.rmtree(stale)


def save_checkpoint(output, model, optimizer, scheduler, step: int, keep_checkpoints: int,
                    meta: Optional[Dict] = None) -> Path:
    d = Path(output) / f"step_{step:07d}"
    d.mkdir(parents=True, exist_ok=True)
    torch.save({k: v.detach().cpu() for k, v in model.state_dict().items()}, d / "model.pt")
    (d / "meta.json").write_text(json.dumps({"step": step, **(meta or {})}, indent=2))
    torch.save({"step": step, "optimizer": optimizer.state_dict(),
                "scheduler": scheduler.state_dict()}, d / ".training_state.tmp")
    (d / ".training_state.tmp").replace(d / "training_state.pt")  # written last
    prune_checkpoints(output, keep_checkpoints)
    return d


def latest_checkpoint(output) -> Optional[Path]:
    done = [p for p in Path(output).glob("step_*") if (p / "training_state.pt").exists()]
    return max(done, key=lambda p: int(p.name[5:])) if done else None


class PromptResponseTarDataset(torch.utils.data.Dataset):
    def __init__(self, tar_path: str, image_size: int = 224,
                 default_prompt: str = DEFAULT_PROMPT):
        self.tar_path, self.size, self.default_prompt = tar_path, image_size, default_prompt
        groups: Dict[str, Dict[str, tarfile.TarInfo]] = {}
        with tarfile.open(tar_path) as tf:
            for m in tf.getmembers():
                if m.isfile() and "." in m.name:
                    k, ext = m.name.rsplit(".", 1)
                    groups.setdefault(k, {})[ext.lower()] = m
        self.items = [(k, g) for k, g in sorted(groups.items())
                      if "txt" in g and any(e in g for e in ("jpg", "jpeg", "png"))]
        self._tf = None

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        import numpy as np
        from PIL import Image

        if self._tf is None:
            self._tf = tarfile.open(self.tar_path)
        k, g = self.items[i]
        m = next(g[e] for e in ("jpg", "jpeg", "png") if e in g)
        img = Image.open(io.BytesIO(self._tf.extractfile(m).read())).convert("RGB")
        img = img.resize((self.size, self.size))
        x = torch.from_numpy(np.asarray(img, dtype=np.uint8).copy()).permute(2, 0, 1).float() / 255
        read = lambda ext: self._tf.extractfile(g[ext]).read().decode("utf-8").strip()  # noqa: E731
        return x, (read("prompt") if "prompt" in g else self.default_prompt), read("txt")


def collate_prompt_response(batch):
    return (torch.stack([b[0] for b in batch]), [b[1] for b in batch], [b[2] for b in batch])


@dataclass
class VLMTrainConfig:
    max_steps: int = 1000
    sft_steps: int = 0
    gradient_accumulation: int = 1
    max_text_length: int = 256
    learning_rate: float = 1e-4
    weight_decay: float = 0.05
    warmup_steps: int = 100
    min_lr_ratio: float = 0.1
    grad_clip: float = 1.0
    save_steps: int = 500
    keep_checkpoints: int = 4
    log_steps: int = 20
    bf16: bool = True
    output: str = "vlm_run"
    resume: bool = False


def train_vlm(model, tokenizer, batches: Iterable, config: VLMTrainConfig,
              sft_batches: Optional[Iterable] = None) -> Dict:
    """Run ``max_steps`` optimizer steps over (images, prompts, responses) batches
    (re-iterated as needed); the final ``sft_steps`` use ``sft_batches`` (or the
    same stream) with the decoder frozen."""
    from .detection.schedule import cosine_schedule

    c = config
    dev = next(model.parameters()).device
    params = [p for p in model.parameters() if p.requires_grad]
    decay = [p for p in params if p.ndim >= 2]
    no_decay = [p for p in params if p.ndim < 2]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": c.weight_decay},
                             {"params": no_decay, "weight_decay": 0.0}], lr=c.learning_rate)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: cosine_schedule(
        s, warmup_steps=min(c.warmup_steps, c.max_steps), total_steps=c.max_steps,
        min_ratio=c.min_lr_ratio))
    step = 0
    if c.resume:
        ck = latest_checkpoint(c.output)
        if ck is not None:
            model.load_state_dict(torch.load(ck / "model.pt", map_location="cpu"))
            st = torch.load(ck / "training_state.pt", map_location="cpu", weights_only=False)
            opt.load_state_dict(st["optimizer"])
            sched.load_state_dict(st["scheduler"])
            step = st["step"]

    def cycle(src):
        while True:
            n = 0
            for b in src:
                n += 1
                yield b
            if n == 0:
                raise ValueError("empty batch source")

    stream = cycle(batches)
    sft_stream = cycle(sft_batches) if sft_batches is not None else None
    amp = c.bf16 and dev.type == "cuda"
    frozen = None
    log: List[Dict] = []
    while step < c.max_steps:
        in_sft = stage_is_sft(step, total_steps=c.max_steps, sft_steps=c.sft_steps)
        if in_sft and frozen is None:
            frozen = freeze_decoder_for_vision_only_sft(model)
        src = sft_stream if (in_sft and sft_stream is not None) else stream
        model.train()
        opt.zero_grad(set_to_none=True)
        tot = 0.0
        for _ in range(c.gradient_accumulation):
            images, prompts, responses = next(src)
            ids, labels = tokenize_prompt_response(tokenizer, prompts, responses,
                                                   c.max_text_length, dev)
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
                loss = model(images.to(dev, non_blocking=True), ids, labels)["loss"]
            (loss / c.gradient_accumulation).backward()
            tot += float(loss.detach()) / c.gradient_accumulation
        torch.nn.utils.clip_grad_norm_([p for p in model.parameters() if p.requires_grad],
                                       c.grad_clip)
        opt.step()
        sched.step()
        step += 1
        if step % c.log_steps == 0 or step == c.max_steps:
            log.append({"step": step, "loss": tot, "lr": sched.get_last_lr()[0],
                        "stage": "sft" if in_sft else "alignment"})
        if step % c.save_steps == 0 or step == c.max_steps:
            save_checkpoint(c.output, model, opt, sched, step, c.keep_checkpoints,
                            {"stage": "sft" if in_sft else "alignment"})
    return {"steps": step, "log": log, "frozen": frozen}
