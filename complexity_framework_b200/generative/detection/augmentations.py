"""Detection training augmentations on tensors (counterpart:
complexity/generative/detection/augmentations.py; the albumentations backend is
not used).  Every transform maps (image [3, S, S] in [0, 1], target dict with
xyxy ``boxes`` and ``labels``) to the same, keeping boxes consistent and
dropping boxes that become (nearly) empty."""
from __future__ import annotations

import random
from typing import Dict, Sequence, Tuple

import torch
import torch.nn.functional as F

Target = Dict[str, torch.Tensor]


def _keep(t: Target, min_size: float = 2.0) -> Target:
    b = t["boxes"]
    ok = ((b[:, 2] - b[:, 0]) >= min_size) & ((b[:, 3] - b[:, 1]) >= min_size)
    return dict(t, boxes=b[ok], labels=t["labels"][ok])


def horizontal_flip(img: torch.Tensor, t: Target) -> Tuple[torch.Tensor, Target]:
    W = img.shape[-1]
    b = t["boxes"].clone()
    b[:, [0, 2]] = W - t["boxes"][:, [2, 0]]
    return img.flip(-1), dict(t, boxes=b)


def random_scale(img: torch.Tensor, t: Target, lo: float = 0.5, hi: float = 1.5,
                 rng: random.Random = random) -> Tuple[torch.Tensor, Target]:
    """Resize by a random factor, then crop or pad (grey) back to the input size
    at a random offset."""
    C, S, _ = img.shape
    s = rng.uniform(lo, hi)
    n = max(8, int(round(S * s)))
    r = F.interpolate(img[None], size=(n, n), mode="bilinear", align_corners=False)[0]
    out = img.new_full((C, S, S), 0.5)
    b = t["boxes"] * (n / S)
    if n >= S:
        ox, oy = rng.randint(0, n - S), rng.randint(0, n - S)
        out = r[:, oy:oy + S, ox:ox + S]
        b = b - torch.tensor([ox, oy, ox, oy], dtype=b.dtype)
    else:
        ox, oy = rng.randint(0, S - n), rng.randint(0, S - n)
        out[:, oy:oy + n, ox:ox + n] = r
        b = b + torch.tensor([ox, oy, ox, oy], dtype=b.dtype)
    return out, _keep(dict(t, boxes=b.clamp(0, S)))


def color_jitter(img: torch.Tensor, t: Target, strength: float = 0.3,
                 rng: random.Random = random) -> Tuple[torch.Tensor, Target]:
    """Brightness, contrast and per-channel gain."""
    b = 1 + rng.uniform(-strength, strength)
    c = 1 + rng.uniform(-strength, strength)
    gain = torch.tensor([1 + rng.uniform(-strength, strength) / 2 for _ in range(img.shape[0])])
    m = img.mean()
    out = ((img - m) * c + m) * b * gain[:, None, None]
    return out.clamp(0, 1), t


def mosaic(samples: Sequence[Tuple[torch.Tensor, Target]],
           rng: random.Random = random) -> Tuple[torch.Tensor, Target]:
    """Four images in the quadrants around a random centre of one canvas of the
    same size (each scaled to half size)."""
    assert len(samples) == 4
    C, S, _ = samples[0][0].shape
    h = S // 2
    canvas = samples[0][0].new_full((C, S, S), 0.5)
    cx, cy = rng.randint(S // 4, 3 * S // 4), rng.randint(S // 4, 3 * S // 4)
    boxes, labels = [], []
    for k, (img, t) in enumerate(samples):
        small = F.interpolate(img[None], size=(h, h), mode="bilinear", align_corners=False)[0]
        x0 = cx - h if k % 2 == 0 else cx
        y0 = cy - h if k < 2 else cy
        xs, ys = max(0, x0), max(0, y0)
        xe, ye = min(S, x0 + h), min(S, y0 + h)
        canvas[:, ys:ye, xs:xe] = small[:, ys - y0:ye - y0, xs - x0:xe - x0]
        b = t["boxes"] * 0.5 + torch.tensor([x0, y0, x0, y0], dtype=torch.float32)
        b[:, [0, 2]] = b[:, [0, 2]].clamp(xs, xe)
        b[:, [1, 3]] = b[:, [1, 3]].clamp(ys, ye)
        boxes.append(b)
        labels.append(t["labels"])
    return canvas, _keep({"boxes": torch.cat(boxes), "labels": torch.cat(labels)})


class DetectionAugment:
    """Mosaic (probability ``p_mosaic``, needs the dataset), flip, scale and colour."""

    def __init__(self, dataset=None, p_mosaic: float = 0.5, p_flip: float = 0.5,
                 scale: Tuple[float, float] = (0.6, 1.4), color: float = 0.3, seed: int = 0):
        self.ds, self.p_mosaic, self.p_flip = dataset, p_mosaic, p_flip
        self.scale, self.color = scale, color
        self.rng = random.Random(seed)

    def __call__(self, img: torch.Tensor, t: Target) -> Tuple[torch.Tensor, Target]:
        r = self.rng
        if self.ds is not None and r.random() < self.p_mosaic:
            others = [self.ds[r.randrange(len(self.ds))] for _ in range(3)]
            img, t = mosaic([(img, t)] + others, r)
        if r.random() < self.p_flip:
            img, t = horizontal_flip(img, t)
        img, t = random_scale(img, t, *self.scale, rng=r)
        return color_jitter(img, t, self.color, r)


class AugmentedDataset(torch.utils.data.Dataset):
    def __init__(self, dataset, augment: DetectionAugment):
        self.ds, self.aug = dataset, augment
        if augment.ds is None:
            augment.ds = dataset

    def __len__(self):
        return len(self.ds)

    def __getitem__(self, i):
        return self.aug(*self.ds[i])
