"""Text cleaning, composable pipelines, token-level augmentation and mixup
collation (counterpart of complexity/data/preprocessing.py:17-380).

``TextPreprocessor`` strips HTML tags, URLs and e-mail addresses, collapses
whitespace, optionally lowercases, drops texts shorter than ``min_length``
and truncates at ``max_length``.  ``DataAugmenter`` deletes, swaps adjacent
and duplicates tokens with independent probabilities (from its own seeded
generator, not the global ``random`` state).  ``MixupCollator`` returns each
batch with a permuted partner batch and a Beta(alpha, alpha) weight for
models that mix in embedding space.
"""
from __future__ import annotations

import random
import re
from typing import Any, Callable, Dict, List, Optional

import torch

_URL = re.compile(r"https?://\S+|www\.\S+")
_EMAIL = re.compile(r"[\w.\-]+@[\w.\-]+\.\w+")
_HTML = re.compile(r"<[^>]+>")
_WS = re.compile(r"\s+")


class TextPreprocessor:
    def __init__(self, lowercase: bool = False, remove_urls: bool = True,
                 remove_emails: bool = True, normalize_whitespace: bool = True,
                 remove_html: bool = True, min_length: int = 10,
                 max_length: Optional[int] = None):
        self.lowercase, self.remove_urls, self.remove_emails = lowercase, remove_urls, remove_emails
        self.normalize_whitespace, self.remove_html = normalize_whitespace, remove_html
        self.min_length, self.max_length = min_length, max_length

    def __call__(self, text: str) -> Optional[str]:
        if not text:
            return None
        for on, pat in ((self.remove_html, _HTML), (self.remove_urls, _URL),
                        (self.remove_emails, _EMAIL)):
            if on:
                text = pat.sub(" ", text)
        if self.normalize_whitespace:
            text = _WS.sub(" ", text).strip()
        if self.lowercase:
            text = text.lower()
        if len(text) < self.min_length:
            return None
        return text[:self.max_length] if self.max_length else text


class DataPipeline:
    """Steps applied in order; a step returning None drops the item."""

    def __init__(self, steps: List[Callable[[Any], Any]]):
        self.steps = list(steps)

    def __call__(self, data: Any) -> Optional[Any]:
        for step in self.steps:
            if data is None:
                return None
            data = step(data)
        return data

    def add_step(self, step: Callable[[Any], Any]) -> None:
        self.steps.append(step)

    @classmethod
    def create_default(cls) -> "DataPipeline":
        return cls([TextPreprocessor()])


class DataAugmenter:
    def __init__(self, delete_prob: float = 0.0, swap_prob: float = 0.0,
                 insert_prob: float = 0.0, seed: Optional[int] = None):
        self.delete_prob, self.swap_prob, self.insert_prob = delete_prob, swap_prob, insert_prob
        self.rng = random.Random(seed)

    def augment_tokens(self, tokens: List[int], seed: Optional[int] = None) -> List[int]:
        r = random.Random(seed) if seed is not None else self.rng
        t = list(tokens)
        if self.delete_prob > 0:
            t = [x for x in t if r.random() > self.delete_prob]
        if self.swap_prob > 0:
            for i in range(len(t) - 1):
                if r.random() < self.swap_prob:
                    t[i], t[i + 1] = t[i + 1], t[i]
        if self.insert_prob > 0:
            out = []
            for x in t:
                out.append(x)
                if r.random() < self.insert_prob:
                    out.append(x)
            t = out
        return t

    def __call__(self, item: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return {"input_ids": torch.tensor(self.augment_tokens(item["input_ids"].tolist()),
                                          dtype=torch.long)}


class MixupCollator:
    def __init__(self, alpha: float = 0.2):
        self.alpha = alpha

    def __call__(self, batch: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
        ids = torch.stack([b["input_ids"] for b in batch])
        labels = torch.stack([b["labels"] for b in batch])
        lam = torch.distributions.Beta(self.alpha, self.alpha).sample()
        perm = torch.randperm(ids.shape[0])
        return {"input_ids": ids, "input_ids_mixed": ids[perm], "labels": labels,
                "labels_mixed": labels[perm], "mixup_lambda": lam}
