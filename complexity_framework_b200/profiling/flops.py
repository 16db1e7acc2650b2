"""FLOP accounting for TR-Hash decoders and arbitrary modules."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Optional

import torch
import torch.nn as nn


def count_parameters(model: nn.Module, trainable_only: bool = False) -> int:
    return sum(p.numel() for p in model.parameters() if p.requires_grad or not trainable_only)


def parameter_breakdown(model: nn.Module) -> Dict[str, int]:
    out: Dict[str, int] = {}
    for name, p in model.named_parameters():
        key = name.split(".")[0] if not name.startswith("layers.") else ".".join(
            name.split(".")[2:3] or ["layers"])
        out[key] = out.get(key, 0) + p.numel()
    return out


def model_flops_per_token(config, seq_len: int, *, training: bool = True,
                          causal: bool = True) -> Dict[str, float]:
    """Matmul FLOPs per token of a TR-Hash decoder (``ModelConfig``).

    Counts what the kernels execute with the *active* routed width (top-k of
    E experts), the attention score/value products (halved when causal) and
    the LM head; training = 3x forward (forward, data grad, weight grad).
    """
    H = config.hidden_size
    L = config.num_hidden_layers
    hq = config.num_attention_heads
    hkv = config.num_key_value_heads or hq
    d = H // hq
    V = config.vocab_size
    shared = getattr(config, "shared_intermediate_size", 0) or 0
    E = max(1, getattr(config, "num_experts", 1) or 1)
    k = min(E, getattr(config, "top_k", 1) or 1)
    w = (getattr(config, "intermediate_size", 0) or 0) // E if E > 1 else 0
    proj = 2 * H * (hq * d + 2 * hkv * d) + 2 * hq * d * H
    attn = 2 * 2 * seq_len * hq * d * (0.5 if causal else 1.0)
    mlp = 2 * 3 * H * shared + 2 * 3 * H * w * k
    head = 2 * H * V
    fwd = L * (proj + attn + mlp) + head
    mult = 3.0 if training else 1.0
    return {"forward": fwd, "total": fwd * mult, "attention": L * attn * mult,
            "dense": (fwd - L * attn) * mult}


def estimate_transformer_flops(num_layers: int, hidden_size: int, seq_len: int, vocab_size: int,
                               batch_size: int = 1, intermediate_size: Optional[int] = None,
                               num_heads: Optional[int] = None, training: bool = True) -> Dict:
    """Generic dense-transformer estimate (Kaplan-style 2*N plus attention)."""
    inter = intermediate_size or 4 * hidden_size
    per_layer = 2 * (4 * hidden_size * hidden_size + 3 * hidden_size * inter) \
        + 2 * 2 * seq_len * hidden_size
    fwd = (num_layers * per_layer + 2 * hidden_size * vocab_size) * seq_len * batch_size
    total = fwd * (3 if training else 1)
    return {"forward_flops": fwd, "total_flops": total, "tflops": total / 1e12}


def profile_model_flops(model: nn.Module, batch_size: int = 1, seq_len: int = 2048) -> Dict:
    n = count_parameters(model)
    t = batch_size * seq_len
    return {"num_params": n, "tokens_per_step": t, "flops_forward": 2 * n * t,
            "flops_total": 6 * n * t, "tflops_total": 6 * n * t / 1e12}


@dataclass
class ModelComplexity:
    flops: int
    params: int
    by_module: Dict[str, int]

    def __str__(self) -> str:
        return f"{self.flops / 1e9:.2f} GFLOPs, {self.params / 1e6:.2f} M params"


class FLOPSCounter:
    """Forward hooks that count matmul FLOPs of Linear / Embedding-free modules
    and of ``TRHashEngine`` layers (active routed width) for one forward."""

    def __init__(self):
        self.by_module: Dict[str, int] = {}
        self._hooks = []

    def reset(self) -> None:
        self.by_module = {}

    def _hook(self, name):
        def fn(mod, inp, out):
            f = self._flops(mod, inp, out)
            if f:
                self.by_module[name] = self.by_module.get(name, 0) + f
        return fn

    @staticmethod
    def _flops(mod, inp, out) -> int:
        x = inp[0] if inp else None
        if isinstance(mod, nn.Linear) and torch.is_tensor(x):
            return 2 * (x.numel() // x.shape[-1]) * mod.in_features * mod.out_features
        if type(mod).__name__ == "TRHashEngine" and torch.is_tensor(x):
            cfg = mod.config
            t = x.numel() // x.shape[-1]
            return t * 2 * 3 * cfg.hidden_size * cfg.active_mlp_width
        if isinstance(mod, (nn.Conv1d, nn.Conv2d)) and torch.is_tensor(out):
            k = mod.weight[0].numel()
            return 2 * out.numel() * k
        return 0

    def count(self, model: nn.Module, *args, **kwargs) -> ModelComplexity:
        self.reset()
        for name, m in model.named_modules():
            if ".engine." in name:
                continue  # the engine hook counts its shared and routed GEMMs
            if isinstance(m, (nn.Linear, nn.Conv1d, nn.Conv2d)) or type(m).__name__ == "TRHashEngine":
                self._hooks.append(m.register_forward_hook(self._hook(name)))
        try:
            with torch.no_grad():
                model(*args, **kwargs)
        finally:
            for h in self._hooks:
                h.remove()
            self._hooks = []
        return ModelComplexity(sum(self.by_module.values()), count_parameters(model),
                               dict(self.by_module))

    def report(self) -> str:
        tot = sum(self.by_module.values()) or 1
        rows = sorted(self.by_module.items(), key=lambda kv: -kv[1])[:20]
        return "\n".join(f"{n:60s} {f / 1e9:10.3f} GF {100 * f / tot:5.1f}%" for n, f in rows)
