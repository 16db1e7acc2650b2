"""Weight quantization: int8 / int4 group-wise / FP8 linear layers and the
dynamic / static quantizers.

Counterpart of complexity/quantization/quantizer.py:20-420.  On B200 the FP8
path is the native one: ``LinearFP8`` stores e4m3 weights with per-row
scales and runs ``torch._scaled_mm`` (the FP8 tensor-core GEMM) on CUDA with
per-token activation scales; elsewhere it dequantises.  Int8 / int4 layers
keep packed weights plus scales and dequantise to the activation dtype.
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Dict, Iterable, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class QuantizationMethod(Enum):
    DYNAMIC = "dynamic"
    STATIC = "static"
    GPTQ = "gptq"
    AWQ = "awq"
    FP8 = "fp8"
    GGUF = "gguf"


@dataclass
class QuantizationConfig:
    bits: int = 8
    method: str = "dynamic"
    group_size: int = 128
    sym: bool = True
    exclude_layers: Optional[List[str]] = None
    calibration_samples: int = 128
    desc_act: bool = True


def quantize_tensor_groupwise(w: torch.Tensor, bits: int, group_size: int, sym: bool = True):
    """Per-(row, group) min/max quantisation of a 2-D weight.

    Returns integer codes (int8 storage), scales and zero points of shape
    ``[rows, ngroups]``.
    """
    rows, cols = w.shape
    g = group_size if group_size > 0 else cols
    pad = (-cols) % g
    wf = F.pad(w.float(), (0, pad)).view(rows, -1, g)
    qmax = 2 ** (bits - 1) - 1 if sym else 2 ** bits - 1
    if sym:
        scale = wf.abs().amax(-1).clamp_min(1e-8) / qmax
        zero = torch.zeros_like(scale)
        q = torch.round(wf / scale[..., None]).clamp(-qmax - 1, qmax)
    else:
        lo, hi = wf.amin(-1), wf.amax(-1)
        scale = (hi - lo).clamp_min(1e-8) / qmax
        zero = torch.round(-lo / scale)
        q = (torch.round(wf / scale[..., None]) + zero[..., None]).clamp(0, qmax)
    return q.to(torch.int8).view(rows, -1)[:, :cols].contiguous(), scale, zero


def dequantize_groupwise(q: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor,
                         group_size: int, dtype=torch.float32) -> torch.Tensor:
    rows, cols = q.shape
    g = group_size if group_size > 0 else cols
    pad = (-cols) % g
    qf = F.pad(q.float(), (0, pad)).view(rows, -1, g)
    w = (qf - zero[..., None]) * scale[..., None]
    return w.view(rows, -1)[:, :cols].to(dtype)


class Linear8bit(nn.Module):
    """int8 weights with per-output-channel scales (weight-only)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.register_buffer("weight_q", torch.zeros(out_features, in_features, dtype=torch.int8))
        self.register_buffer("scale", torch.ones(out_features))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None

    @classmethod
    def from_linear(cls, lin: nn.Linear) -> "Linear8bit":
        m = cls(lin.in_features, lin.out_features, lin.bias is not None)
        w = lin.weight.detach().float()
        s = w.abs().amax(1).clamp_min(1e-8) / 127
        m.weight_q.copy_(torch.round(w / s[:, None]).clamp(-128, 127).to(torch.int8))
        m.scale.copy_(s)
        if lin.bias is not None:
            m.bias.data.copy_(lin.bias.detach())
        return m.to(lin.weight.device)

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        return (self.weight_q.float() * self.scale[:, None]).to(dtype)

    def forward(self, x):
        return F.linear(x, self.dequantize(x.dtype), self.bias)


class Linear4bit(nn.Module):
    """Group-wise 4-bit weights, two codes per byte."""

    def __init__(self, in_features: int, out_features: int, group_size: int = 128,
                 bias: bool = False, sym: bool = True):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.group_size, self.sym = group_size, sym
        ng = -(-in_features // group_size)
        self.register_buffer("packed", torch.zeros(out_features, (in_features + 1) // 2,
                                                   dtype=torch.uint8))
        self.register_buffer("scale", torch.ones(out_features, ng))
        self.register_buffer("zero", torch.zeros(out_features, ng))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None

    @staticmethod
    def pack(q: torch.Tensor, sym: bool) -> torch.Tensor:
        u = (q.to(torch.int16) + (8 if sym else 0)).to(torch.uint8)
        if u.shape[1] % 2:
            u = F.pad(u, (0, 1))
        return (u[:, 0::2] | (u[:, 1::2] << 4)).contiguous()

    def unpack(self) -> torch.Tensor:
        lo = (self.packed & 0xF).to(torch.int16)
        hi = (self.packed >> 4).to(torch.int16)
        q = torch.stack((lo, hi), -1).view(self.out_features, -1)[:, :self.in_features]
        return (q - 8) if self.sym else q

    @classmethod
    def from_linear(cls, lin: nn.Linear, group_size: int = 128, sym: bool = True) -> "Linear4bit":
        m = cls(lin.in_features, lin.out_features, group_size, lin.bias is not None, sym)
        q, s, z = quantize_tensor_groupwise(lin.weight.detach(), 4, group_size, sym)
        m.packed.copy_(cls.pack(q, sym))
        m.scale.copy_(s)
        m.zero.copy_(z)
        if lin.bias is not None:
            m.bias.data.copy_(lin.bias.detach())
        return m.to(lin.weight.device)

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        return dequantize_groupwise(self.unpack(), self.scale, self.zero, self.group_size, dtype)

    def forward(self, x):
        return F.linear(x, self.dequantize(x.dtype), self.bias)


_FP8 = getattr(torch, "float8_e4m3fn", None)
_FP8_MAX = 448.0


class LinearFP8(nn.Module):
    """e4m3 weights with per-output-row scales.  CUDA: per-token dynamic
    activation scaling and ``torch._scaled_mm`` on the FP8 tensor cores."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        if _FP8 is None:
            raise RuntimeError("this torch build has no float8_e4m3fn")
        self.in_features, self.out_features = in_features, out_features
        self.register_buffer("weight_fp8", torch.zeros(out_features, in_features, dtype=_FP8))
        self.register_buffer("scale", torch.ones(out_features))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None

    @classmethod
    def from_linear(cls, lin: nn.Linear) -> "LinearFP8":
        m = cls(lin.in_features, lin.out_features, lin.bias is not None)
        w = lin.weight.detach().float()
        s = w.abs().amax(1).clamp_min(1e-12) / _FP8_MAX
        m.weight_fp8.copy_((w / s[:, None]).to(_FP8))
        m.scale.copy_(s)
        if lin.bias is not None:
            m.bias.data.copy_(lin.bias.detach())
        return m.to(lin.weight.device)

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        return (self.weight_fp8.float() * self.scale[:, None]).to(dtype)

    def forward(self, x):
        shp = x.shape
        if x.is_cuda and hasattr(torch, "_scaled_mm") and self.in_features % 16 == 0 \
                and self.out_features % 16 == 0:
            x2 = x.reshape(-1, shp[-1])
            xs = x2.float().abs().amax(1, keepdim=True).clamp_min(1e-12) / _FP8_MAX
            xq = (x2.float() / xs).to(_FP8)
            y = torch._scaled_mm(xq, self.weight_fp8.t(), scale_a=xs,
                                 scale_b=self.scale[None, :].float(), out_dtype=x.dtype)
            if self.bias is not None:
                y = y + self.bias
            return y.view(*shp[:-1], self.out_features)
        return F.linear(x, self.dequantize(x.dtype), self.bias)


def _replace_linears(model: nn.Module, make, exclude: Iterable[str] = ()) -> int:
    n = 0
    excl = list(exclude or [])
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            full = f"{name}.{cname}" if name else cname
            if isinstance(child, nn.Linear) and not any(e in full for e in excl):
                setattr(mod, cname, make(child))
                n += 1
    return n


class DynamicQuantizer:
    """Weight-only quantisation of every ``nn.Linear`` (8, 4 bit, or FP8)."""

    def __init__(self, config: QuantizationConfig):
        self.config = config

    def quantize(self, model: nn.Module) -> nn.Module:
        c = self.config
        excl = c.exclude_layers or ["lm_head"]
        if c.method == "fp8":
            make = LinearFP8.from_linear
        elif c.bits == 8:
            make = Linear8bit.from_linear
        elif c.bits == 4:
            make = lambda l: Linear4bit.from_linear(l, c.group_size, c.sym)  # noqa: E731
        else:
            raise ValueError("bits must be 4 or 8")
        _replace_linears(model, make, excl)
        return model


class StaticQuantizer(DynamicQuantizer):
    """Calibrated int8: activation ranges are recorded on calibration batches
    and stored per layer (``act_scale``) next to the int8 weights."""

    def calibrate(self, model: nn.Module, batches: Iterable[torch.Tensor]) -> Dict[str, float]:
        ranges: Dict[str, float] = {}
        hooks = []
        for name, m in model.named_modules():
            if isinstance(m, nn.Linear):
                def hook(mod, inp, out, name=name):
                    ranges[name] = max(ranges.get(name, 0.0), float(inp[0].detach().abs().max()))
                hooks.append(m.register_forward_hook(hook))
        with torch.no_grad():
            for i, b in enumerate(batches):
                if i >= self.config.calibration_samples:
                    break
                model(b)
        for h in hooks:
            h.remove()
        self.ranges = ranges
        return ranges

    def quantize(self, model: nn.Module) -> nn.Module:
        ranges = getattr(self, "ranges", {})
        model = super().quantize(model)
        for name, m in model.named_modules():
            if name in ranges and hasattr(m, "scale"):
                m.register_buffer("act_scale", torch.tensor(ranges[name] / 127.0))
        return model


def quantize_model(model: nn.Module, config: Optional[QuantizationConfig] = None, bits: int = 8,
                   method: str = "dynamic", calibration_data=None, **kwargs) -> nn.Module:
    cfg = config or QuantizationConfig(bits=bits, method=method, **kwargs)
    if cfg.method in ("dynamic", "fp8"):
        return DynamicQuantizer(cfg).quantize(model)
    if cfg.method == "static":
        q = StaticQuantizer(cfg)
        if calibration_data is not None:
            q.calibrate(model, calibration_data)
        return q.quantize(model)
    if cfg.method == "gptq":
        from .gptq import GPTQConfig, gptq_quantize_model

        return gptq_quantize_model(model, calibration_data, GPTQConfig(bits=cfg.bits,
                                                                       group_size=cfg.group_size))
    if cfg.method == "awq":
        from .awq import AWQConfig, awq_quantize

        return awq_quantize(model, calibration_data, AWQConfig(bits=cfg.bits,
                                                               group_size=cfg.group_size))
    raise ValueError(f"unknown quantization method {cfg.method!r}")


def get_model_size(model: nn.Module) -> Dict[str, float]:
    tot = sum(t.numel() * t.element_size() for t in list(model.parameters()) + list(model.buffers()))
    return {"bytes": tot, "mb": tot / 2 ** 20}


@torch.no_grad()
def compare_outputs(a: nn.Module, b: nn.Module, inputs) -> Dict[str, float]:
    oa, ob = a(inputs), b(inputs)
    oa = oa["logits"] if isinstance(oa, dict) else oa
    ob = ob["logits"] if isinstance(ob, dict) else ob
    d = (oa.float() - ob.float())
    return {"max_abs": float(d.abs().max()), "mse": float(d.pow(2).mean()),
            "cosine": float(F.cosine_similarity(oa.float().flatten(), ob.float().flatten(), 0))}
