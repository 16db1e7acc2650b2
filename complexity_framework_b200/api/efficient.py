"""Small-budget helpers: quantisation, mixed precision, memory savers and
small model presets.

Facade names follow complexity/api/core/efficient.py (``QuantConfig``,
``Quantize``, ``QuantizedLinear``, ``MixedPrecision``, ``MemoryEfficient``,
``SmallModels``, ``Efficient``).  Quantised layers are this framework's own
(``quantization/``: int8 / int4 group-wise, FP8 on ``torch._scaled_mm``).
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Dict, Iterable, Optional

import torch
import torch.nn as nn

from ..config.model_config import ModelConfig
from ..quantization.quantizer import (Linear4bit, Linear8bit, LinearFP8, QuantizationConfig,
                                      quantize_model)


@dataclass
class QuantConfig:
    bits: int = 8                 # 8, 4, or 8 with fp8=True
    group_size: int = 128
    symmetric: bool = True
    fp8: bool = False
    exclude: tuple = ("lm_head", "embed_tokens")

    def to_internal(self) -> QuantizationConfig:
        return QuantizationConfig(bits=self.bits, method="fp8" if self.fp8 else "dynamic",
                                  group_size=self.group_size, sym=self.symmetric,
                                  exclude_layers=list(self.exclude))


class QuantizedLinear(nn.Module):
    """A quantised drop-in for ``nn.Linear`` (int8, int4 group-wise, or FP8)."""

    def __init__(self, inner: nn.Module):
        super().__init__()
        self.inner = inner

    @classmethod
    def from_linear(cls, linear: nn.Linear, config: Optional[QuantConfig] = None) -> "QuantizedLinear":
        c = config or QuantConfig()
        if c.fp8:
            q = LinearFP8.from_linear(linear)
        elif c.bits == 4:
            q = Linear4bit.from_linear(linear, group_size=c.group_size)
        else:
            q = Linear8bit.from_linear(linear)
        return cls(q)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.inner(x)


class Quantize:
    @staticmethod
    def dynamic(model: nn.Module, bits: int = 8, **kwargs) -> nn.Module:
        return quantize_model(model, QuantConfig(bits=bits, **kwargs).to_internal())

    @staticmethod
    def static(model: nn.Module, calibration_data: Optional[Iterable[torch.Tensor]] = None,
               bits: int = 4, method: str = "gptq", **kwargs) -> nn.Module:
        """Calibrated weight-only quantisation (``gptq`` or ``awq``)."""
        if method == "awq":
            from ..quantization.awq import AWQConfig, awq_quantize

            return awq_quantize(model, calibration_data, AWQConfig(bits=bits, **kwargs))
        from ..quantization.gptq import GPTQConfig, gptq_quantize_model

        return gptq_quantize_model(model, calibration_data, GPTQConfig(bits=bits, **kwargs))

    @staticmethod
    def linear(linear: nn.Linear, bits: int = 8, **kwargs) -> nn.Module:
        return QuantizedLinear.from_linear(linear, QuantConfig(bits=bits, **kwargs))

    @staticmethod
    def estimate_savings(model: nn.Module, bits: int = 4) -> Dict[str, str]:
        n = sum(p.numel() for p in model.parameters())
        cur = sum(p.numel() * p.element_size() for p in model.parameters())
        new = n * bits / 8
        return {"parameters": f"{n:,}", "current": f"{cur / 2**20:.1f} MiB",
                "quantized": f"{new / 2**20:.1f} MiB", "ratio": f"{cur / max(new, 1):.2f}x"}


class MixedPrecision:
    @staticmethod
    def setup(dtype: str = "bf16") -> torch.dtype:
        return {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]

    @staticmethod
    def autocast(dtype: str = "bf16", device_type: str = "cuda"):
        if device_type == "cuda" and not torch.cuda.is_available():
            return contextlib.nullcontext()
        return torch.autocast(device_type, dtype=MixedPrecision.setup(dtype))

    @staticmethod
    def backward(loss: torch.Tensor, scaler: Optional["torch.amp.GradScaler"] = None) -> None:
        (scaler.scale(loss) if scaler is not None else loss).backward()

    @staticmethod
    def convert_to_fp16(model: nn.Module) -> nn.Module:
        return model.half()

    @staticmethod
    def convert_to_bf16(model: nn.Module) -> nn.Module:
        return model.to(torch.bfloat16)


class MemoryEfficient:
    @staticmethod
    def enable_checkpointing(model: nn.Module) -> nn.Module:
        if hasattr(model, "gradient_checkpointing_enable"):
            model.gradient_checkpointing_enable()
        return model

    @staticmethod
    def disable_checkpointing(model: nn.Module) -> nn.Module:
        if hasattr(model, "gradient_checkpointing_disable"):
            model.gradient_checkpointing_disable()
        return model

    @staticmethod
    def accumulate(model: nn.Module, micro_batches, loss_fn) -> torch.Tensor:
        """Sum of ``loss_fn(model, mb) / n`` with one backward per micro-batch."""
        mbs = list(micro_batches)
        total = None
        for mb in mbs:
            loss = loss_fn(model, mb) / len(mbs)
            loss.backward()
            total = loss.detach() if total is None else total + loss.detach()
        return total

    @staticmethod
    def estimate(model: nn.Module, batch_size: int = 1, seq_len: int = 2048,
                 optimizer: str = "adamw") -> Dict[str, str]:
        """Bytes for weights (bf16), fp32 master + Adam moments, and activations
        (a rough 34 * B * S * H per layer)."""
        n = sum(p.numel() for p in model.parameters())
        cfg = getattr(model, "config", None)
        H = getattr(cfg, "hidden_size", 0)
        L = getattr(cfg, "num_hidden_layers", 0)
        weights = 2 * n
        opt = 12 * n if optimizer == "adamw" else 4 * n
        act = 34 * batch_size * seq_len * H * L
        gib = 2 ** 30
        return {"weights": f"{weights / gib:.2f} GiB", "optimizer": f"{opt / gib:.2f} GiB",
                "activations": f"{act / gib:.2f} GiB",
                "total": f"{(weights + opt + act) / gib:.2f} GiB"}

    @staticmethod
    def offload_to_cpu(model: nn.Module) -> nn.Module:
        return model.cpu()

    @staticmethod
    def clear_cache() -> None:
        if torch.cuda.is_available():
            torch.cuda.empty_cache()


class SmallModels:
    """TR-Hash models for small budgets (GQA, shared SwiGLU + 4 routed experts)."""

    SIZES = {
        "nano": dict(hidden_size=128, num_hidden_layers=4, num_attention_heads=4,
                     num_key_value_heads=2, intermediate_size=256, shared_intermediate_size=384),
        "micro": dict(hidden_size=256, num_hidden_layers=6, num_attention_heads=4,
                      num_key_value_heads=2, intermediate_size=512, shared_intermediate_size=768),
        "tiny": dict(hidden_size=384, num_hidden_layers=8, num_attention_heads=6,
                     num_key_value_heads=2, intermediate_size=768, shared_intermediate_size=1152),
        "small": dict(hidden_size=512, num_hidden_layers=12, num_attention_heads=8,
                      num_key_value_heads=2, intermediate_size=1024, shared_intermediate_size=1536),
        "medium": dict(hidden_size=768, num_hidden_layers=16, num_attention_heads=12,
                       num_key_value_heads=4, intermediate_size=1536,
                       shared_intermediate_size=2304),
    }

    @classmethod
    def config(cls, size: str, vocab_size: int = 32000, **kwargs) -> ModelConfig:
        kw = dict(cls.SIZES[size], vocab_size=vocab_size, num_experts=4, top_k=2,
                  routing_strategy="token_id_multi_hash", max_position_embeddings=2048)
        kw.update(kwargs)
        return ModelConfig(**kw)

    @classmethod
    def create(cls, size: str = "tiny", vocab_size: int = 32000, **kwargs) -> nn.Module:
        from ..models.builder import ComplexityModel

        return ComplexityModel(cls.config(size, vocab_size, **kwargs))

    @classmethod
    def nano(cls, vocab_size: int = 32000, **kwargs) -> nn.Module:
        return cls.create("nano", vocab_size, **kwargs)

    @classmethod
    def micro(cls, vocab_size: int = 32000, **kwargs) -> nn.Module:
        return cls.create("micro", vocab_size, **kwargs)

    @classmethod
    def tiny(cls, vocab_size: int = 32000, **kwargs) -> nn.Module:
        return cls.create("tiny", vocab_size, **kwargs)

    @classmethod
    def small(cls, vocab_size: int = 32000, **kwargs) -> nn.Module:
        return cls.create("small", vocab_size, **kwargs)

    @classmethod
    def medium(cls, vocab_size: int = 32000, **kwargs) -> nn.Module:
        return cls.create("medium", vocab_size, **kwargs)

    @classmethod
    def estimate_params(cls, size: str, vocab_size: int = 32000) -> str:
        from ..profiling.flops import count_parameters

        n = count_parameters(cls.create(size, vocab_size))
        return f"{n / 1e6:.1f}M"


class Efficient:
    QuantConfig = QuantConfig
    Quantize = Quantize
    QuantizedLinear = QuantizedLinear
    MixedPrecision = MixedPrecision
    MemoryEfficient = MemoryEfficient
    SmallModels = SmallModels

    @staticmethod
    def quantize_model(model: nn.Module, bits: int = 4) -> nn.Module:
        return Quantize.dynamic(model, bits=bits)

    @staticmethod
    def mixed_precision(dtype: str = "bf16", device_type: str = "cuda"):
        return MixedPrecision.autocast(dtype, device_type)

    @staticmethod
    def enable_checkpointing(model: nn.Module) -> nn.Module:
        return MemoryEfficient.enable_checkpointing(model)

    @staticmethod
    def estimate_memory(model: nn.Module, batch_size: int = 1, seq_len: int = 2048) -> Dict[str, str]:
        return MemoryEfficient.estimate(model, batch_size, seq_len)

    @staticmethod
    def estimate_savings(model: nn.Module, bits: int = 4) -> Dict[str, str]:
        return Quantize.estimate_savings(model, bits)

    @staticmethod
    def nano_llm(vocab_size: int = 32000, **kwargs) -> nn.Module:
        return SmallModels.nano(vocab_size, **kwargs)

    @staticmethod
    def micro_llm(vocab_size: int = 32000, **kwargs) -> nn.Module:
        return SmallModels.micro(vocab_size, **kwargs)

    @staticmethod
    def tiny_llm(vocab_size: int = 32000, **kwargs) -> nn.Module:
        return SmallModels.tiny(vocab_size, **kwargs)

    @staticmethod
    def small_llm(vocab_size: int = 32000, **kwargs) -> nn.Module:
        return SmallModels.small(vocab_size, **kwargs)


__all__ = ["QuantConfig", "Quantize", "QuantizedLinear", "MixedPrecision", "MemoryEfficient",
           "SmallModels", "Efficient"]
