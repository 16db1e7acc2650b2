"""Low-rank adapters (LoRA) for dense and stacked-expert weights.

Counterpart of complexity/training/lora.py:22-339 (``LoRALinear``,
``LoRAExpertTensor`` as a parametrisation of ``[E, in, out]`` expert stacks,
adapter state dicts, merge/unmerge).

Design: adapters are weight parametrisations, ``W_eff = W + s * B A`` (dense
``[out, in]``) or ``W_eff = W + s * A_e B_e`` per expert (``[E, in, out]``,
one batched matmul).  Every module keeps its parameter names and shapes, so
the fused sm_100a kernels, the weight packing and the checkpoint format are
unchanged: the kernels simply read ``W_eff``.  The low-rank product is one
tiny GEMM per adapted weight per step.  ``LoRALinear`` is the module-wrapper
form (input-side dropout on the low-rank path) for code that wants it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Sequence

import torch
import torch.nn as nn
from torch.nn.utils import parametrize

DEFAULT_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "shared_gate", "shared_up",
                   "shared_down")
EXPERT_TARGETS = ("expert_gate", "expert_up", "expert_down")


@dataclass
class LoRAConfig:
    r: int = 8
    alpha: float = 16.0
    dropout: float = 0.0
    target_modules: Sequence[str] = field(default_factory=lambda: list(DEFAULT_TARGETS))
    include_experts: bool = False
    train_norms: bool = False

    @property
    def scale(self) -> float:
        return self.alpha / self.r


class LoRADelta(nn.Module):
    """Parametrisation of a dense ``[out, in]`` weight: ``W + scale * B @ A``."""

    def __init__(self, out_features: int, in_features: int, r: int, scale: float,
                 device=None, dtype=None):
        super().__init__()
        self.lora_A = nn.Parameter(torch.empty(r, in_features, device=device, dtype=dtype))
        self.lora_B = nn.Parameter(torch.zeros(out_features, r, device=device, dtype=dtype))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.scale = scale
        self.enabled = True

    def forward(self, W: torch.Tensor) -> torch.Tensor:
        if not self.enabled:
            return W
        return W + (self.lora_B @ self.lora_A).to(W.dtype) * self.scale


class LoRAExpertTensor(nn.Module):
    """Parametrisation of an expert stack ``[E, in, out]``: ``W_e + scale * A_e @ B_e``."""

    def __init__(self, num_experts: int, in_features: int, out_features: int, r: int,
                 scale: float, device=None, dtype=None):
        super().__init__()
        self.lora_A = nn.Parameter(torch.empty(num_experts, in_features, r, device=device,
                                               dtype=dtype))
        self.lora_B = nn.Parameter(torch.zeros(num_experts, r, out_features, device=device,
                                               dtype=dtype))
        nn.init.normal_(self.lora_A, std=1.0 / math.sqrt(in_features))
        self.scale = scale
        self.enabled = True

    def forward(self, W: torch.Tensor) -> torch.Tensor:
        if not self.enabled:
            return W
        return torch.baddbmm(W, self.lora_A.to(W.dtype), self.lora_B.to(W.dtype),
                             alpha=self.scale)


class LoRALinear(nn.Module):
    """Wrapper form: ``y = base(x) + scale * dropout(x) A^T B^T``; ``merge``
    folds the update into ``base.weight`` and ``unmerge`` takes it out again."""

    def __init__(self, base: nn.Linear, r: int = 8, alpha: float = 16.0, dropout: float = 0.0):
        super().__init__()
        self.base = base
        self.r = r
        self.scale = alpha / r
        dev, dt = base.weight.device, base.weight.dtype
        self.lora_A = nn.Parameter(torch.empty(r, base.in_features, device=dev, dtype=dt))
        self.lora_B = nn.Parameter(torch.zeros(base.out_features, r, device=dev, dtype=dt))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.merged = False
        self.enabled = True
        base.weight.requires_grad_(False)

    @property
    def weight(self) -> torch.Tensor:
        return self.base.weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.base(x)
        if self.merged or not self.enabled:
            return y
        return y + (self.dropout(x) @ self.lora_A.t() @ self.lora_B.t()) * self.scale

    @torch.no_grad()
    def merge(self) -> None:
        if not self.merged:
            self.base.weight += (self.lora_B @ self.lora_A) * self.scale
            self.merged = True

    @torch.no_grad()
    def unmerge(self) -> None:
        if self.merged:
            self.base.weight -= (self.lora_B @ self.lora_A) * self.scale
            self.merged = False


def _targets(name: str, cfg: LoRAConfig) -> bool:
    leaf = name.split(".")[-1]
    return leaf in cfg.target_modules


def apply_lora(model: nn.Module, config: Optional[LoRAConfig] = None) -> List[str]:
    """Freeze the base model and attach adapters.  Returns the adapted weight names."""
    cfg = config or LoRAConfig()
    for n, p in model.named_parameters():
        p.requires_grad_(cfg.train_norms and "norm" in n)
    adapted = []
    for mname, mod in list(model.named_modules()):
        if isinstance(mod, nn.Linear) and _targets(mname, cfg):
            W = mod.weight
            parametrize.register_parametrization(
                mod, "weight", LoRADelta(W.shape[0], W.shape[1], cfg.r, cfg.scale, W.device,
                                         W.dtype))
            adapted.append(f"{mname}.weight")
        if cfg.include_experts:
            for pname in EXPERT_TARGETS:
                W = getattr(mod, "_parameters", {}).get(pname)
                if W is not None and W.ndim == 3:
                    parametrize.register_parametrization(
                        mod, pname, LoRAExpertTensor(W.shape[0], W.shape[1], W.shape[2], cfg.r,
                                                     cfg.scale, W.device, W.dtype))
                    adapted.append(f"{mname}.{pname}")
    for n, p in model.named_parameters():
        if ".parametrizations." in n and "original" in n:
            p.requires_grad_(False)
    return adapted


def lora_parameters(model: nn.Module) -> List[nn.Parameter]:
    return [p for n, p in model.named_parameters() if "lora_" in n]


def lora_state_dict(model: nn.Module) -> Dict[str, torch.Tensor]:
    """Adapter weights only (what an SFT run saves)."""
    return {n: p.detach().cpu() for n, p in model.named_parameters() if "lora_" in n}


def load_lora_state_dict(model: nn.Module, sd: Dict[str, torch.Tensor]) -> None:
    own = dict(model.named_parameters())
    missing = [k for k in sd if k not in own]
    if missing:
        raise KeyError(f"adapter keys not in model: {missing[:4]}")
    with torch.no_grad():
        for k, v in sd.items():
            own[k].copy_(v)


def set_lora_enabled(model: nn.Module, enabled: bool) -> None:
    for m in model.modules():
        if isinstance(m, (LoRADelta, LoRAExpertTensor, LoRALinear)):
            m.enabled = enabled


def merge_lora(model: nn.Module) -> int:
    """Fold every adapter into its base weight and drop the parametrisations
    (the model's state dict is then the plain checkpoint format).  Returns the
    number of merged weights."""
    count = 0
    for mod in list(model.modules()):
        if parametrize.is_parametrized(mod):
            for pname in list(mod.parametrizations.keys()):
                parametrize.remove_parametrizations(mod, pname, leave_parametrized=True)
                count += 1
        if isinstance(mod, LoRALinear):
            mod.merge()
            count += 1
    return count


def count_trainable(model: nn.Module) -> Dict[str, int]:
    tot = sum(p.numel() for p in model.parameters())
    tr = sum(p.numel() for p in model.parameters() if p.requires_grad)
    return {"total": tot, "trainable": tr}


# ------------------------------------------------- reference adapter helpers
# complexity/training/lora.py:234-339 names adapters by their module (dense)
# or "<module>.<expert tensor>" (stacked experts) and keeps adapter-only state
# dicts under "<name>.lora_A" / "<name>.lora_B"; the same names are used here
# for both the parametrised weights and the LoRALinear wrapper.
def lora_modules(model: nn.Module) -> Dict[str, nn.Module]:
    """Dense adapters by module name (LoRALinear wrappers and LoRADelta weights)."""
    out: Dict[str, nn.Module] = {}
    for name, mod in model.named_modules():
        if isinstance(mod, LoRALinear):
            out[name] = mod
        elif parametrize.is_parametrized(mod, "weight"):
            p = mod.parametrizations["weight"]
            if len(p) == 1 and isinstance(p[0], LoRADelta):
                out[name] = p[0]
    return out


def expert_lora_modules(model: nn.Module):
    """``{"<module>.<tensor>": (parent, tensor name, LoRAExpertTensor)}``."""
    out = {}
    for name, mod in model.named_modules():
        if not parametrize.is_parametrized(mod):
            continue
        for tname, plist in mod.parametrizations.items():
            if len(plist) == 1 and isinstance(plist[0], LoRAExpertTensor):
                out[f"{name}.{tname}" if name else tname] = (mod, tname, plist[0])
    return out


def adapter_state_dict(model: nn.Module) -> Dict[str, torch.Tensor]:
    st = {}
    for name, m in lora_modules(model).items():
        st[f"{name}.lora_A"], st[f"{name}.lora_B"] = m.lora_A.detach().cpu(), m.lora_B.detach().cpu()
    for name, (_, _, m) in expert_lora_modules(model).items():
        st[f"{name}.lora_A"], st[f"{name}.lora_B"] = m.lora_A.detach().cpu(), m.lora_B.detach().cpu()
    return st


def load_adapter_state_dict(model: nn.Module, state: Dict[str, torch.Tensor]) -> None:
    """Load adapter weights; the key set must match this model's adapters exactly."""
    mods = {**lora_modules(model), **{k: v[2] for k, v in expert_lora_modules(model).items()}}
    expected = {f"{n}.{p}" for n in mods for p in ("lora_A", "lora_B")}
    if set(state) != expected:
        miss, extra = sorted(expected - set(state)), sorted(set(state) - expected)
        raise ValueError(f"adapter state does not match the model's adapters "
                         f"(missing {miss[:4]}, unexpected {extra[:4]})")
    with torch.no_grad():
        for n, m in mods.items():
            m.lora_A.copy_(state[f"{n}.lora_A"])
            m.lora_B.copy_(state[f"{n}.lora_B"])


def _delta(m: nn.Module) -> torch.Tensor:
    if isinstance(m, LoRAExpertTensor):
        return torch.bmm(m.lora_A, m.lora_B) * m.scale
    return (m.lora_B @ m.lora_A) * m.scale


def unmerge_adapter_from_base(model: nn.Module) -> None:
    """Given base weights that already contain the adapters' update, subtract it
    so base + adapter is again the merged model (the inverse of merging)."""
    with torch.no_grad():
        for name, m in lora_modules(model).items():
            if isinstance(m, LoRALinear):
                m.base.weight.sub_(_delta(m).to(m.base.weight.dtype))
            else:
                owner = model.get_submodule(name)
                orig = owner.parametrizations["weight"].original
                orig.sub_(_delta(m).to(orig.dtype))
        for parent, tname, m in expert_lora_modules(model).values():
            orig = parent.parametrizations[tname].original
            orig.sub_(_delta(m).to(orig.dtype))


def merged_model_state_dict(model: nn.Module) -> Dict[str, torch.Tensor]:
    """The plain checkpoint state (adapters folded in) without changing ``model``."""
    out: Dict[str, torch.Tensor] = {}
    dense = lora_modules(model)
    experts = expert_lora_modules(model)
    for key, val in model.state_dict().items():
        if key.endswith(".lora_A") or key.endswith(".lora_B"):
            continue
        if ".parametrizations." in key:
            owner, rest = key.split(".parametrizations.", 1)
            tname = rest.split(".")[0]
            if not rest.endswith(".original"):
                continue
            a = dense.get(owner) if tname == "weight" else None
            e = experts.get(f"{owner}.{tname}")
            m = a if a is not None else (e[2] if e is not None else None)
            out[f"{owner}.{tname}"] = (val + _delta(m).to(val.dtype)).detach() if m is not None \
                else val
            continue
        if key.endswith(".base.weight") and key[:-len(".base.weight")] in dense:
            m = dense[key[:-len(".base.weight")]]
            w = val if getattr(m, "merged", False) else val + _delta(m).to(val.dtype)
            out[key[:-len(".base.weight")] + ".weight"] = w.detach()
            continue
        if ".base." in key and key.split(".base.")[0] in dense:
            out[key.replace(".base.", ".")] = val
            continue
        out[key] = val
    return out
