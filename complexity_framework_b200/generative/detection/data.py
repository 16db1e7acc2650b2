"""Detection data: class-name tables, letterbox pre/post-processing, a synthetic
shapes dataset and the batch collate.

Counterparts: complexity/generative/detection/data.py (``COCO_CLASS_NAMES``,
``VOC_CLASS_NAMES``, ``SyntheticShapesDataset``, ``collate_detection``,
``preprocess_detector_image``, ``restore_detector_boxes``,
``DetectionImageMetadata``) and the COCO / YOLO-format datasets, which read
annotation files from disk (``CocoDetectionDataset``, ``YoloDetectionDataset``).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch
import torch.nn.functional as F

COCO_CLASS_NAMES = (
    "person", "bicycle", "car", "motorcycle", "airplane", "bus", "train", "truck", "boat",
    "traffic light", "fire hydrant", "stop sign", "parking meter", "bench", "bird", "cat", "dog",
    "horse", "sheep", "cow", "elephant", "bear", "zebra", "giraffe", "backpack", "umbrella",
    "handbag", "tie", "suitcase", "frisbee", "skis", "snowboard", "sports ball", "kite",
    "baseball bat", "baseball glove", "skateboard", "surfboard", "tennis racket", "bottle",
    "wine glass", "cup", "fork", "knife", "spoon", "bowl", "banana", "apple", "sandwich",
    "orange", "broccoli", "carrot", "hot dog", "pizza", "donut", "cake", "chair", "couch",
    "potted plant", "bed", "dining table", "toilet", "tv", "laptop", "mouse", "remote",
    "keyboard", "cell phone", "microwave", "oven", "toaster", "sink", "refrigerator", "book",
    "clock", "vase", "scissors", "teddy bear", "hair drier", "toothbrush")
VOC_CLASS_NAMES = (
    "aeroplane", "bicycle", "bird", "boat", "bottle", "bus", "car", "cat", "chair", "cow",
    "diningtable", "dog", "horse", "motorbike", "person", "pottedplant", "sheep", "sofa",
    "train", "tvmonitor")


@dataclass
class DetectionImageMetadata:
    """How an image was letterboxed: ``scale`` then padding ``(pad_x, pad_y)``."""
    original_size: Tuple[int, int]   # (height, width)
    scale: float
    pad_x: float
    pad_y: float


def preprocess_detector_image(image: torch.Tensor, size: int
                              ) -> Tuple[torch.Tensor, DetectionImageMetadata]:
    """[C, H, W] float image in [0, 1] -> letterboxed [C, size, size] (aspect kept,
    grey padding centred) and the metadata to map boxes back."""
    C, H, W = image.shape
    s = size / max(H, W)
    nh, nw = max(1, round(H * s)), max(1, round(W * s))
    img = F.interpolate(image[None], size=(nh, nw), mode="bilinear", align_corners=False)[0]
    out = image.new_full((C, size, size), 0.5)
    py, px = (size - nh) // 2, (size - nw) // 2
    out[:, py:py + nh, px:px + nw] = img
    return out, DetectionImageMetadata((H, W), s, float(px), float(py))


def restore_detector_boxes(boxes: torch.Tensor, meta: DetectionImageMetadata) -> torch.Tensor:
    """Letterboxed xyxy boxes -> original image coordinates (clipped)."""
    b = boxes.clone()
    b[:, [0, 2]] = (b[:, [0, 2]] - meta.pad_x) / meta.scale
    b[:, [1, 3]] = (b[:, [1, 3]] - meta.pad_y) / meta.scale
    H, W = meta.original_size
    b[:, [0, 2]] = b[:, [0, 2]].clamp(0, W)
    b[:, [1, 3]] = b[:, [1, 3]].clamp(0, H)
    return b


class SyntheticShapesDataset(torch.utils.data.Dataset):
    """Filled rectangles (class 0) and ellipses (class 1), optionally more classes
    by colour, on a noisy background: a self-contained detection task."""

    def __init__(self, length: int = 256, image_size: int = 128, max_objects: int = 4,
                 num_classes: int = 2, seed: int = 0):
        self.length, self.size, self.max_obj, self.nc, self.seed = (length, image_size,
                                                                   max_objects, num_classes, seed)

    def __len__(self) -> int:
        return self.length

    def __getitem__(self, i: int):
        g = torch.Generator().manual_seed(self.seed * 1000003 + i)
        S = self.size
        img = 0.1 * torch.rand(3, S, S, generator=g)
        n = int(torch.randint(1, self.max_obj + 1, (1,), generator=g))
        boxes, labels = [], []
        yy, xx = torch.meshgrid(torch.arange(S), torch.arange(S), indexing="ij")
        for _ in range(n):
            w, h = (torch.randint(S // 8, S // 3, (2,), generator=g)).tolist()
            x0 = int(torch.randint(0, S - w, (1,), generator=g))
            y0 = int(torch.randint(0, S - h, (1,), generator=g))
            cls = int(torch.randint(0, self.nc, (1,), generator=g))
            colour = torch.tensor([(cls + 1) % 3 == 0, (cls + 1) % 3 == 1, (cls + 1) % 3 == 2],
                                  dtype=torch.float32) * 0.8 + 0.2
            if cls % 2 == 0:
                m = (xx >= x0) & (xx < x0 + w) & (yy >= y0) & (yy < y0 + h)
            else:
                cx, cy = x0 + w / 2, y0 + h / 2
                m = ((xx - cx) / (w / 2)) ** 2 + ((yy - cy) / (h / 2)) ** 2 <= 1
            img[:, m] = colour[:, None]
            boxes.append([x0, y0, x0 + w, y0 + h])
            labels.append(cls)
        return img, {"boxes": torch.tensor(boxes, dtype=torch.float32),
                     "labels": torch.tensor(labels, dtype=torch.long)}


def collate_detection(batch: Sequence) -> Tuple[torch.Tensor, List[Dict[str, torch.Tensor]]]:
    images = torch.stack([b[0] for b in batch])
    return images, [b[1] for b in batch]


class CocoDetectionDataset(torch.utils.data.Dataset):
    """COCO-format annotations (``instances_*.json``) with images in ``image_dir``;
    images are letterboxed to ``image_size``.  Categories map to contiguous labels."""

    def __init__(self, annotation_file: str, image_dir: str, image_size: int = 640):
        with open(annotation_file) as f:
            ann = json.load(f)
        self.image_dir, self.size = image_dir, image_size
        self.cat_ids = sorted(c["id"] for c in ann["categories"])
        self.cat_to_label = {c: i for i, c in enumerate(self.cat_ids)}
        self.images = ann["images"]
        self.by_image: Dict[int, list] = {}
        for a in ann["annotations"]:
            if not a.get("iscrowd", 0):
                self.by_image.setdefault(a["image_id"], []).append(a)

    def __len__(self) -> int:
        return len(self.images)

    def _read(self, path: str) -> torch.Tensor:
        from torchvision.io import read_image  # optional dependency

        return read_image(path).float() / 255.0

    def __getitem__(self, i: int):
        info = self.images[i]
        img = self._read(os.path.join(self.image_dir, info["file_name"]))
        img, meta = preprocess_detector_image(img, self.size)
        boxes, labels = [], []
        for a in self.by_image.get(info["id"], []):
            x, y, w, h = a["bbox"]
            boxes.append([x * meta.scale + meta.pad_x, y * meta.scale + meta.pad_y,
                          (x + w) * meta.scale + meta.pad_x, (y + h) * meta.scale + meta.pad_y])
            labels.append(self.cat_to_label[a["category_id"]])
        return img, {"boxes": torch.tensor(boxes, dtype=torch.float32).reshape(-1, 4),
                     "labels": torch.tensor(labels, dtype=torch.long), "image_id": info["id"],
                     "meta": meta}


class YoloDetectionDataset(torch.utils.data.Dataset):
    """YOLO text labels (``class cx cy w h`` normalised, one file per image)."""

    def __init__(self, image_dir: str, label_dir: str, image_size: int = 640):
        self.image_dir, self.label_dir, self.size = image_dir, label_dir, image_size
        self.files = sorted(f for f in os.listdir(image_dir)
                            if f.lower().endswith((".jpg", ".jpeg", ".png")))

    def __len__(self) -> int:
        return len(self.files)

    def __getitem__(self, i: int):
        from torchvision.io import read_image  # optional dependency

        name = self.files[i]
        img = read_image(os.path.join(self.image_dir, name)).float() / 255.0
        H, W = img.shape[-2:]
        img, meta = preprocess_detector_image(img, self.size)
        boxes, labels = [], []
        lp = os.path.join(self.label_dir, os.path.splitext(name)[0] + ".txt")
        if os.path.exists(lp):
            for line in open(lp):
                p = line.split()
                if len(p) < 5:
                    continue
                c, cx, cy, w, h = int(p[0]), *map(float, p[1:5])
                x0, y0 = (cx - w / 2) * W, (cy - h / 2) * H
                boxes.append([x0 * meta.scale + meta.pad_x, y0 * meta.scale + meta.pad_y,
                              (x0 + w * W) * meta.scale + meta.pad_x,
                              (y0 + h * H) * meta.scale + meta.pad_y])
                labels.append(c)
        return img, {"boxes": torch.tensor(boxes, dtype=torch.float32).reshape(-1, 4),
                     "labels": torch.tensor(labels, dtype=torch.long), "meta": meta}
