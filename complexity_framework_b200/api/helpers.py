"""Helper namespaces: initialisation, masks, KV caches, sampling, tensor
utilities, debugging and checkpointing.

Facade names and call shapes follow complexity/api/core/helpers.py (``Init``,
``Mask``, ``KVCache``, ``SlidingWindowCache``, ``Sampling``, ``Tensors``,
``Debug``, ``Checkpointing``, ``Helpers``).
"""
from __future__ import annotations

import math
from pathlib import Path
from typing import Dict, List, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..core.layers import apply_rotary_pos_emb, rotate_half


class Init:
    """Weight initialisers applied to every Linear / Embedding of a module."""

    @staticmethod
    def apply(module: nn.Module, method: str = "normal", **kwargs) -> nn.Module:
        fn = {"normal": Init.normal, "xavier": Init.xavier, "kaiming": Init.kaiming,
              "orthogonal": Init.orthogonal, "zeros": Init.zeros}[method]
        return fn(module, **kwargs)

    @staticmethod
    def _weights(module: nn.Module):
        for m in module.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                yield m

    @staticmethod
    @torch.no_grad()
    def normal(module: nn.Module, std: float = 0.02, **kwargs) -> nn.Module:
        for m in Init._weights(module):
            m.weight.normal_(0.0, std)
            if getattr(m, "bias", None) is not None:
                m.bias.zero_()
        return module

    @staticmethod
    @torch.no_grad()
    def xavier(module: nn.Module, gain: float = 1.0, **kwargs) -> nn.Module:
        for m in Init._weights(module):
            nn.init.xavier_uniform_(m.weight, gain=gain)
        return module

    @staticmethod
    @torch.no_grad()
    def kaiming(module: nn.Module, mode: str = "fan_in", nonlinearity: str = "relu",
                **kwargs) -> nn.Module:
        for m in Init._weights(module):
            nn.init.kaiming_normal_(m.weight, mode=mode, nonlinearity=nonlinearity)
        return module

    @staticmethod
    @torch.no_grad()
    def orthogonal(module: nn.Module, gain: float = 1.0, **kwargs) -> nn.Module:
        for m in Init._weights(module):
            nn.init.orthogonal_(m.weight, gain=gain)
        return module

    @staticmethod
    @torch.no_grad()
    def zeros(module: nn.Module, **kwargs) -> nn.Module:
        for m in Init._weights(module):
            m.weight.zero_()
        return module

    @staticmethod
    @torch.no_grad()
    def scaled_init(module: nn.Module, num_layers: int, std: float = 0.02) -> nn.Module:
        """Output projections (o_proj, *down*) scaled by 1/sqrt(2 * num_layers)."""
        scale = std / math.sqrt(2.0 * num_layers)
        for name, m in module.named_modules():
            if isinstance(m, nn.Linear) and ("o_proj" in name or "down" in name):
                m.weight.normal_(0.0, scale)
        return module


class Mask:
    """Additive attention masks ([.., q, kv], 0 = attend, -inf = masked)."""

    @staticmethod
    def causal(seq_len: int, device=None, dtype=torch.float32,
               kv_len: Optional[int] = None) -> torch.Tensor:
        kv = kv_len or seq_len
        q = torch.arange(kv - seq_len, kv, device=device)[:, None]
        k = torch.arange(kv, device=device)[None, :]
        return torch.zeros(seq_len, kv, device=device, dtype=dtype).masked_fill(k > q, float("-inf"))

    @staticmethod
    def padding(attention_mask: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
        """[B, S] 1/0 -> [B, 1, 1, S] additive."""
        m = attention_mask[:, None, None, :].to(dtype)
        return (1.0 - m) * torch.finfo(dtype).min

    @staticmethod
    def sliding_window(seq_len: int, window: int, device=None,
                       dtype=torch.float32) -> torch.Tensor:
        q = torch.arange(seq_len, device=device)[:, None]
        k = torch.arange(seq_len, device=device)[None, :]
        bad = (k > q) | (q - k >= window)
        return torch.zeros(seq_len, seq_len, device=device, dtype=dtype).masked_fill(bad, float("-inf"))

    @staticmethod
    def block_sparse(seq_len: int, block_size: int, num_global_blocks: int = 1, device=None,
                     dtype=torch.float32) -> torch.Tensor:
        """Causal; each query sees its own block, the previous one and the first
        ``num_global_blocks`` blocks."""
        q = torch.arange(seq_len, device=device)[:, None] // block_size
        k = torch.arange(seq_len, device=device)[None, :] // block_size
        ok = ((q - k) <= 1) | (k < num_global_blocks)
        ok &= torch.arange(seq_len, device=device)[None, :] <= torch.arange(seq_len, device=device)[:, None]
        return torch.zeros(seq_len, seq_len, device=device, dtype=dtype).masked_fill(~ok, float("-inf"))

    @staticmethod
    def combine(*masks: torch.Tensor) -> torch.Tensor:
        out = masks[0]
        for m in masks[1:]:
            out = out + m
        return out


class KVCache:
    """Per-layer contiguous K/V cache ``[B, Hkv, S, D]`` grown by ``update``."""

    def __init__(self, num_layers: int):
        self.k: List[Optional[torch.Tensor]] = [None] * num_layers
        self.v: List[Optional[torch.Tensor]] = [None] * num_layers

    @classmethod
    def create(cls, num_layers: int, **kwargs) -> "KVCache":
        return cls(num_layers)

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor):
        if self.k[layer_idx] is None:
            self.k[layer_idx], self.v[layer_idx] = k, v
        else:
            self.k[layer_idx] = torch.cat([self.k[layer_idx], k], dim=2)
            self.v[layer_idx] = torch.cat([self.v[layer_idx], v], dim=2)
        return self.k[layer_idx], self.v[layer_idx]

    def get(self, layer_idx: int) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        return self.k[layer_idx], self.v[layer_idx]

    def clear(self) -> None:
        self.k = [None] * len(self.k)
        self.v = [None] * len(self.v)

    @property
    def seq_length(self) -> int:
        return 0 if self.k[0] is None else self.k[0].shape[2]


class SlidingWindowCache(KVCache):
    """KV cache that keeps only the last ``window`` positions."""

    def __init__(self, num_layers: int, window: int = 4096):
        super().__init__(num_layers)
        self.window = window

    @classmethod
    def create(cls, num_layers: int, window: int = 4096, **kwargs) -> "SlidingWindowCache":
        return cls(num_layers, window)

    def update(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor):
        kk, vv = super().update(layer_idx, k, v)
        if kk.shape[2] > self.window:
            self.k[layer_idx] = kk[:, :, -self.window:].contiguous()
            self.v[layer_idx] = vv[:, :, -self.window:].contiguous()
        return self.k[layer_idx], self.v[layer_idx]


class Sampling:
    @staticmethod
    def temperature(logits: torch.Tensor, t: float = 1.0) -> torch.Tensor:
        return logits / max(t, 1e-6)

    @staticmethod
    def top_k(logits: torch.Tensor, k: int = 50) -> torch.Tensor:
        if k <= 0 or k >= logits.shape[-1]:
            return logits
        kth = torch.topk(logits, k, dim=-1).values[..., -1:]
        return logits.masked_fill(logits < kth, float("-inf"))

    @staticmethod
    def top_p(logits: torch.Tensor, p: float = 0.9) -> torch.Tensor:
        if p >= 1.0:
            return logits
        sorted_l, idx = torch.sort(logits, descending=True, dim=-1)
        probs = sorted_l.softmax(-1)
        drop = probs.cumsum(-1) - probs > p
        sorted_l = sorted_l.masked_fill(drop, float("-inf"))
        return torch.full_like(logits, float("-inf")).scatter(-1, idx, sorted_l)

    @staticmethod
    def greedy(logits: torch.Tensor) -> torch.Tensor:
        return logits.argmax(-1)

    @staticmethod
    def sample(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
               generator: Optional[torch.Generator] = None) -> torch.Tensor:
        if temperature <= 0:
            return Sampling.greedy(logits)
        x = Sampling.top_p(Sampling.top_k(Sampling.temperature(logits.float(), temperature),
                                          top_k), top_p)
        probs = x.softmax(-1)
        flat = probs.reshape(-1, probs.shape[-1])
        out = torch.multinomial(flat, 1, generator=generator).view(probs.shape[:-1])
        return out


class Tensors:
    @staticmethod
    def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
        """[B, Hkv, S, D] -> [B, Hkv * n_rep, S, D]."""
        return x if n_rep == 1 else x.repeat_interleave(n_rep, dim=1)

    @staticmethod
    def rotate_half(x: torch.Tensor) -> torch.Tensor:
        return rotate_half(x)

    @staticmethod
    def apply_rotary(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        return apply_rotary_pos_emb(q, k, cos, sin)

    @staticmethod
    def chunk(x: torch.Tensor, num_chunks: int, dim: int = 0) -> List[torch.Tensor]:
        return list(torch.chunk(x, num_chunks, dim=dim))

    @staticmethod
    def interleave(tensors: List[torch.Tensor], dim: int = 0) -> torch.Tensor:
        return torch.stack(tensors, dim=dim + 1).flatten(dim, dim + 1)


class Debug:
    @staticmethod
    def count_params(model: nn.Module, trainable_only: bool = False) -> Dict[str, int]:
        total = sum(p.numel() for p in model.parameters())
        train = sum(p.numel() for p in model.parameters() if p.requires_grad)
        return {"total": train if trainable_only else total, "trainable": train,
                "frozen": total - train}

    @staticmethod
    def model_summary(model: nn.Module, max_depth: int = 2) -> str:
        lines = []
        for name, m in model.named_modules():
            depth = name.count(".") + (1 if name else 0)
            if depth > max_depth:
                continue
            n = sum(p.numel() for p in m.parameters())
            lines.append(f"{'  ' * depth}{name or type(m).__name__}: {type(m).__name__} "
                         f"({n:,} params)")
        return "\n".join(lines)

    @staticmethod
    def memory_usage(device: Union[str, torch.device] = "cuda") -> Dict[str, str]:
        if not torch.cuda.is_available():
            return {"allocated": "0 B", "reserved": "0 B", "peak": "0 B"}
        d = torch.device(device)
        gib = 1024 ** 3
        return {"allocated": f"{torch.cuda.memory_allocated(d) / gib:.2f} GiB",
                "reserved": f"{torch.cuda.memory_reserved(d) / gib:.2f} GiB",
                "peak": f"{torch.cuda.max_memory_allocated(d) / gib:.2f} GiB"}

    @staticmethod
    def print_summary(model: nn.Module, max_depth: int = 2) -> None:
        print(Debug.model_summary(model, max_depth))


class Checkpointing:
    """Activation checkpointing switches and weight save/load helpers."""

    @staticmethod
    def enable(model: nn.Module) -> nn.Module:
        if hasattr(model, "gradient_checkpointing_enable"):
            model.gradient_checkpointing_enable()
        return model

    @staticmethod
    def disable(model: nn.Module) -> nn.Module:
        if hasattr(model, "gradient_checkpointing_disable"):
            model.gradient_checkpointing_disable()
        return model

    @staticmethod
    def save(model: nn.Module, path: Union[str, Path]) -> None:
        model.save_pretrained(path)

    @staticmethod
    def load(path: Union[str, Path]):
        from ..models.builder import ComplexityModel

        return ComplexityModel.from_pretrained(path)


class Helpers:
    Init = Init
    Mask = Mask
    KVCache = KVCache
    SlidingWindowCache = SlidingWindowCache
    Sampling = Sampling
    Tensors = Tensors
    Debug = Debug
    Checkpointing = Checkpointing


__all__ = ["Init", "Mask", "KVCache", "SlidingWindowCache", "Sampling", "Tensors", "Debug",
           "Checkpointing", "Helpers"]
