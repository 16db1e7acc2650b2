"""Optimizer family beyond the fused AdamW: Muon, MuonTR, AdamTR, MuSGD, Lion,
Sophia, 8-bit Adam, CAME, AdaLomo, and the ``get_optimizer`` factory.

Counterparts: complexity/training/muon.py:20-330 (Newton-Schulz, ``Muon``,
``MuonWithAdamW``, ``split_params_for_muon``), muon_tr.py:45-600 (``MuonTR``
per-expert orthogonalisation), adam_tr.py:101-400 (``AdamTR``), musgd.py:14-170
(``MuSGD``), optimizers.py:30-700 (Lion, Sophia, Adam8bit, CAME, AdaLomo,
``get_optimizer``).

These are ordinary ``torch.optim.Optimizer`` subclasses; the matrix work
(Newton-Schulz iterations) is batched matmuls in bf16 on the tensor cores, one
batched call per expert stack instead of a Python loop over experts.  The
Trainer wraps them with :class:`DistributedOptimizer` for gradient
all-reduce and clipping when it does not use the flat fused AdamW.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch.optim import Optimizer

# Quintic Newton-Schulz coefficients of the public Muon method (K. Jordan et
# al., 2024): they push all singular values of X towards ~1 in few steps.
_NS_COEFFS = (3.4445, -4.7750, 2.0315)


def newton_schulz(M: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Approximate the orthogonal polar factor U V^T of ``M`` (..., rows, cols).

    Batched over leading dimensions; works in bf16 on CUDA (fp32 on CPU).
    """
    a, b, c = _NS_COEFFS
    dtype = torch.bfloat16 if M.is_cuda else torch.float32
    X = M.to(dtype)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = X.transpose(-2, -1)
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + eps)
    for _ in range(steps):
        A = X @ X.transpose(-2, -1)
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if transposed:
        X = X.transpose(-2, -1)
    return X.to(M.dtype)


def zeroth_power_newton_schulz(matrix: torch.Tensor) -> torch.Tensor:
    """Orthogonal factor of one 2-D matrix (five Newton-Schulz steps), the
    MuSGD helper of complexity/training/musgd.py:14."""
    if matrix.ndim != 2:
        raise ValueError("MuSGD orthogonalization expects a 2D matrix")
    return newton_schulz(matrix)


def newton_schulz_adaptive(M: torch.Tensor, min_steps: int = 5, max_steps: int = 10,
                           tol: float = 1e-2, eps: float = 1e-7) -> Tuple[torch.Tensor, int]:
    """Newton-Schulz iterated until the relative change falls under ``tol``.

    Returns ``(X, steps_taken)``.  Used for noisy (low-token) expert slices,
    whose wider singular-value spread needs more iterations.
    """
    a, b, c = _NS_COEFFS
    dtype = torch.bfloat16 if M.is_cuda else torch.float32
    X = M.to(dtype)
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = X.transpose(-2, -1)
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + eps)
    taken = 0
    for i in range(max_steps):
        A = X @ X.transpose(-2, -1)
        Xn = a * X + (b * A + c * (A @ A)) @ X
        taken = i + 1
        delta = (Xn - X).float().norm() / (X.float().norm() + eps)
        X = Xn
        if taken >= min_steps and float(delta) < tol:
            break
    if transposed:
        X = X.transpose(-2, -1)
    return X.to(M.dtype), taken


def _shape_scale(rows: int, cols: int) -> float:
    return math.sqrt(max(1.0, rows / cols))


def _orthogonal_update(update: torch.Tensor, ns_steps: int) -> torch.Tensor:
    shape = update.shape
    u2 = update.reshape(shape[0], -1) if update.ndim > 2 else update
    o = newton_schulz(u2, ns_steps) * _shape_scale(u2.shape[0], u2.shape[1])
    return o.reshape(shape)


class Muon(Optimizer):
    """Momentum + Newton-Schulz orthogonalised updates for >=2-D weights."""

    def __init__(self, params, lr: float = 0.02, momentum: float = 0.95, nesterov: bool = True,
                 ns_steps: int = 5, weight_decay: float = 0.01):
        if lr < 0:
            raise ValueError(f"invalid lr {lr}")
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov,
                                      ns_steps=ns_steps, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if not st:
                    st["momentum_buffer"] = torch.zeros_like(p.grad, dtype=torch.float32)
                buf = st["momentum_buffer"]
                grad = p.grad.float()
                buf.lerp_(grad, 1 - g["momentum"])
                upd = grad.lerp(buf, g["momentum"]) if g["nesterov"] else buf
                o = _orthogonal_update(upd, g["ns_steps"]) if p.ndim >= 2 else upd
                if g["weight_decay"]:
                    p.mul_(1 - g["lr"] * g["weight_decay"])
                p.add_(o.to(p.dtype), alpha=-g["lr"])
        return loss


def split_params_for_muon(model: torch.nn.Module) -> Tuple[List[dict], List[dict]]:
    """Hidden >=2-D weights go to Muon; embeddings, LM head, norms, biases and
    1-D tensors go to AdamW (no decay for norms/biases/embeddings)."""
    muon, adam_decay, adam_nodecay = [], [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        lname = name.lower()
        is_embed = "embed" in lname or "lm_head" in lname
        if p.ndim >= 2 and not is_embed:
            muon.append(p)
        elif p.ndim < 2 or "norm" in lname or "bias" in lname or is_embed:
            adam_nodecay.append(p)
        else:
            adam_decay.append(p)
    adam = []
    if adam_decay:
        adam.append({"params": adam_decay})
    if adam_nodecay:
        adam.append({"params": adam_nodecay, "weight_decay": 0.0})
    return ([{"params": muon}] if muon else []), adam


class MuonWithAdamW(Optimizer):
    """Muon for hidden matrices plus AdamW for everything else, one ``step``."""

    def __init__(self, muon_params, adam_params, lr: float = 0.02, adam_lr: float = 3e-4,
                 momentum: float = 0.95, nesterov: bool = True, ns_steps: int = 5,
                 weight_decay: float = 0.01, adam_betas=(0.9, 0.95), adam_eps: float = 1e-8):
        groups = []
        for g in muon_params:
            g = dict(g)
            g.setdefault("lr", lr)
            g.setdefault("weight_decay", weight_decay)
            g["use_muon"] = True
            groups.append(g)
        for g in adam_params:
            g = dict(g)
            g.setdefault("lr", adam_lr)
            g.setdefault("weight_decay", weight_decay)
            g["use_muon"] = False
            groups.append(g)
        super().__init__(groups, dict(lr=lr, momentum=momentum, nesterov=nesterov,
                                      ns_steps=ns_steps, weight_decay=weight_decay,
                                      betas=adam_betas, eps=adam_eps, use_muon=True))

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                grad = p.grad.float()
                if g["use_muon"]:
                    if not st:
                        st["momentum_buffer"] = torch.zeros_like(grad)
                    buf = st["momentum_buffer"]
                    buf.lerp_(grad, 1 - g["momentum"])
                    upd = grad.lerp(buf, g["momentum"]) if g["nesterov"] else buf
                    o = _orthogonal_update(upd, g["ns_steps"]) if p.ndim >= 2 else upd
                    if g["weight_decay"]:
                        p.mul_(1 - g["lr"] * g["weight_decay"])
                    p.add_(o.to(p.dtype), alpha=-g["lr"])
                else:
                    _adamw_update(p, grad, st, g["lr"], g["betas"], g["eps"], g["weight_decay"])
        return loss


def _adamw_update(p, grad, st, lr, betas, eps, wd, lr_scale: float = 1.0):
    if not st:
        st["step"] = 0
        st["exp_avg"] = torch.zeros_like(grad)
        st["exp_avg_sq"] = torch.zeros_like(grad)
    st["step"] += 1
    b1, b2 = betas
    st["exp_avg"].lerp_(grad, 1 - b1)
    st["exp_avg_sq"].mul_(b2).addcmul_(grad, grad, value=1 - b2)
    bc1 = 1 - b1 ** st["step"]
    bc2 = 1 - b2 ** st["step"]
    denom = (st["exp_avg_sq"] / bc2).sqrt_().add_(eps)
    if wd:
        p.mul_(1 - lr * lr_scale * wd)
    p.add_((st["exp_avg"] / bc1 / denom).to(p.dtype), alpha=-lr * lr_scale)


# ----------------------------------------------------------------- TR variants
def classify_param(name: str, p: torch.Tensor, num_experts: int) -> str:
    """'expert' for stacked routed-expert tensors [E, ...], 'shared' for the
    shared SwiGLU path, 'embed' / 'norm' / 'other' for the rest."""
    lname = name.lower()
    if ("expert_" in lname or ".experts" in lname) and p.ndim == 3 and p.shape[0] == num_experts:
        return "expert"
    if "shared" in lname:
        return "shared"
    if "embed" in lname or "lm_head" in lname:
        return "embed"
    if p.ndim < 2 or "norm" in lname or "bias" in lname:
        return "norm"
    return "other"


def tr_param_groups(model: torch.nn.Module, num_experts: int, *, weight_decay: float = 0.01,
                    expert_weight_decay: float = 0.005) -> List[dict]:
    """Groups tagged with ``param_type`` for :class:`MuonTR` / :class:`AdamTR`."""
    buckets: Dict[str, List] = {}
    for name, p in model.named_parameters():
        if p.requires_grad:
            buckets.setdefault(classify_param(name, p, num_experts), []).append(p)
    out = []
    for kind, ps in buckets.items():
        wd = 0.0 if kind in ("norm", "embed") else (
            expert_weight_decay if kind == "expert" else weight_decay)
        out.append({"params": ps, "param_type": kind, "weight_decay": wd})
    return out


class MuonTR(Optimizer):
    """Muon with per-expert orthogonalisation for token-routed expert stacks.

    An expert tensor [E, a, b] is orthogonalised as E independent matrices in
    one batched Newton-Schulz call.  With ``token_counts`` (tokens per expert)
    the learning rate of expert e is scaled by an EMA of
    sqrt(mean_count / count_e), capped at ``max_lr_ratio`` (tail experts that
    see fewer tokens get larger steps).  A linear warmup ramps the
    orthogonalised step size over ``lr_warmup_steps``.  Non-matrix groups
    (norms, embeddings) use AdamW.
    """

    def __init__(self, params, lr: float = 0.003, momentum: float = 0.95, nesterov: bool = True,
                 ns_steps: int = 5, ns_max_steps: int = 10, ns_tol: float = 1e-4,
                 adaptive_ns: bool = False, weight_decay: float = 0.01,
                 expert_lr_scale: float = 1.0, shared_lr_scale: float = 1.0,
                 expert_weight_decay: float = 0.005, shared_weight_decay: float = 0.01,
                 token_counts: Optional[torch.Tensor] = None, num_experts: int = 4,
                 ema_decay: float = 0.998, max_lr_ratio: float = 2.0, lr_warmup_steps: int = 50,
                 adam_lr: float = 3e-4, adam_betas=(0.9, 0.95), adam_eps: float = 1e-8):
        defaults = dict(lr=lr, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
                        ns_max_steps=ns_max_steps, ns_tol=ns_tol, adaptive_ns=adaptive_ns,
                        weight_decay=weight_decay, param_type="other", adam_lr=adam_lr,
                        betas=adam_betas, eps=adam_eps)
        super().__init__(params, defaults)
        for g in self.param_groups:
            kind = g["param_type"]
            if kind == "expert":
                g.setdefault("lr_scale", expert_lr_scale)
                g["weight_decay"] = g.get("weight_decay", expert_weight_decay)
            elif kind == "shared":
                g.setdefault("lr_scale", shared_lr_scale)
                g["weight_decay"] = g.get("weight_decay", shared_weight_decay)
            else:
                g.setdefault("lr_scale", 1.0)
        self.num_experts = num_experts
        self.ema_decay = ema_decay
        self.max_lr_ratio = max_lr_ratio
        self.lr_warmup_steps = lr_warmup_steps
        self._steps = 0
        self._ratio = None
        if token_counts is not None:
            self.set_token_counts(token_counts)

    def set_token_counts(self, counts: torch.Tensor) -> None:
        c = counts.detach().float().clamp_min(1.0)
        r = (c.mean() / c).sqrt().clamp(max=self.max_lr_ratio)
        self._ratio = r if self._ratio is None else (
            self.ema_decay * self._ratio.to(r.device) + (1 - self.ema_decay) * r)

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._steps += 1
        warm = min(1.0, self._steps / self.lr_warmup_steps) if self.lr_warmup_steps else 1.0
        for g in self.param_groups:
            kind = g["param_type"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                grad = p.grad.float()
                if kind in ("norm", "embed") or p.ndim < 2:
                    _adamw_update(p, grad, st, g["adam_lr"], g["betas"], g["eps"],
                                  g["weight_decay"])
                    continue
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(grad)
                buf = st["momentum_buffer"]
                buf.lerp_(grad, 1 - g["momentum"])
                upd = grad.lerp(buf, g["momentum"]) if g["nesterov"] else buf.clone()
                lr = g["lr"] * g["lr_scale"] * warm
                if kind == "expert" and p.ndim == 3:
                    if g["adaptive_ns"]:
                        o, _ = newton_schulz_adaptive(upd, g["ns_steps"], g["ns_max_steps"],
                                                      g["ns_tol"])
                    else:
                        o = newton_schulz(upd, g["ns_steps"])
                    o = o * _shape_scale(p.shape[1], p.shape[2])
                    scale = torch.full((p.shape[0],), lr, device=p.device)
                    if self._ratio is not None and self._ratio.numel() == p.shape[0]:
                        scale = scale * self._ratio.to(p.device)
                    if g["weight_decay"]:
                        p.mul_((1 - scale * g["weight_decay"]).view(-1, 1, 1).to(p.dtype))
                    p.sub_((o * scale.view(-1, 1, 1)).to(p.dtype))
                else:
                    o = _orthogonal_update(upd, g["ns_steps"])
                    if g["weight_decay"]:
                        p.mul_(1 - lr * g["weight_decay"])
                    p.add_(o.to(p.dtype), alpha=-lr)
        return loss


class MuonTRWithAdamW(MuonTR):
    """Alias kept for API parity: MuonTR already routes non-matrix groups to AdamW."""


def split_params_for_muon_tr(model: torch.nn.Module, num_experts: int = 4, **kw) -> List[dict]:
    return tr_param_groups(model, num_experts, **kw)


def _top_singular(W: torch.Tensor, iters: int = 6) -> torch.Tensor:
    """Largest singular value of each matrix in a [E, a, b] stack (power iteration)."""
    v = torch.ones(W.shape[0], W.shape[2], 1, device=W.device, dtype=torch.float32)
    Wf = W.float()
    for _ in range(iters):
        u = Wf @ v
        u = u / (u.norm(dim=1, keepdim=True) + 1e-12)
        v = Wf.transpose(1, 2) @ u
        v = v / (v.norm(dim=1, keepdim=True) + 1e-12)
    return (Wf @ v).norm(dim=(1, 2))


class AdamTR(Optimizer):
    """AdamW with token-routed awareness.

    * per-kind learning-rate scale and weight decay (``expert_*``, ``shared_*``);
    * optional ``token_counts`` scaling of each expert's step (sqrt(mean/count));
    * spectral conditioning: for an expert stack [E, a, b] the top singular
      value s_e of each expert's update is tracked by an EMA; after
      ``spectral_warmup_steps`` an expert whose s_e exceeds the median is
      scaled down by max(floor, median / s_e), so no single expert's update
      dominates the stack's spectrum.
    """

    def __init__(self, params, lr: float = 3e-4, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.1, expert_lr_scale: float = 1.5,
                 shared_lr_scale: float = 1.0, expert_weight_decay: float = 0.05,
                 shared_weight_decay: float = 0.1, token_counts: Optional[torch.Tensor] = None,
                 num_experts: int = 4, spectral_conditioning: bool = True,
                 spectral_ema: float = 0.99, spectral_floor: float = 0.7,
                 spectral_warmup_steps: int = 50):
        if lr < 0 or eps < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError("invalid AdamTR hyper-parameters")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      param_type="other"))
        for g in self.param_groups:
            if g["param_type"] == "expert":
                g.setdefault("lr_scale", expert_lr_scale)
                g["weight_decay"] = expert_weight_decay
            elif g["param_type"] == "shared":
                g.setdefault("lr_scale", shared_lr_scale)
                g["weight_decay"] = shared_weight_decay
            else:
                g.setdefault("lr_scale", 1.0)
        self.num_experts = num_experts
        self.spectral = spectral_conditioning
        self.spectral_ema = spectral_ema
        self.spectral_floor = spectral_floor
        self.spectral_warmup = spectral_warmup_steps
        self.token_counts = token_counts

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            b1, b2 = g["betas"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                grad = p.grad.float()
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(grad)
                    st["exp_avg_sq"] = torch.zeros_like(grad)
                st["step"] += 1
                st["exp_avg"].lerp_(grad, 1 - b1)
                st["exp_avg_sq"].mul_(b2).addcmul_(grad, grad, value=1 - b2)
                upd = (st["exp_avg"] / (1 - b1 ** st["step"])) / (
                    (st["exp_avg_sq"] / (1 - b2 ** st["step"])).sqrt() + g["eps"])
                lr = g["lr"] * g["lr_scale"]
                if g["param_type"] == "expert" and p.ndim == 3:
                    scale = torch.ones(p.shape[0], device=p.device)
                    if self.token_counts is not None and self.token_counts.numel() == p.shape[0]:
                        c = self.token_counts.float().to(p.device).clamp_min(1)
                        scale = scale * (c.mean() / c).sqrt()
                    if self.spectral:
                        s = _top_singular(upd)
                        ema = st.get("sigma_ema")
                        st["sigma_ema"] = s if ema is None else (
                            self.spectral_ema * ema + (1 - self.spectral_ema) * s)
                        if st["step"] > self.spectral_warmup:
                            e = st["sigma_ema"]
                            scale = scale * (e.median() / e.clamp_min(1e-12)).clamp(
                                self.spectral_floor, 1.0)
                    upd = upd * scale.view(-1, 1, 1)
                if g["weight_decay"]:
                    p.mul_(1 - lr * g["weight_decay"])
                p.add_(upd.to(p.dtype), alpha=-lr)
        return loss


def adamtr_param_groups(model: torch.nn.Module, num_experts: int = 4, **kw) -> List[dict]:
    return tr_param_groups(model, num_experts, **kw)


class MuSGD(Optimizer):
    """SGD with momentum whose matrix updates are orthogonalised (Newton-Schulz)
    and rescaled to the RMS of the raw momentum; vectors take plain momentum SGD."""

    def __init__(self, params, lr: float = 0.01, momentum: float = 0.9, nesterov: bool = True,
                 weight_decay: float = 0.0, ns_steps: int = 5):
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov,
                                      weight_decay=weight_decay, ns_steps=ns_steps))

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                grad = p.grad.float()
                st = self.state[p]
                if not st:
                    st["momentum_buffer"] = torch.zeros_like(grad)
                buf = st["momentum_buffer"]
                buf.mul_(g["momentum"]).add_(grad)
                upd = grad.add(buf, alpha=g["momentum"]) if g["nesterov"] else buf
                if p.ndim >= 2:
                    rms = upd.pow(2).mean().sqrt()
                    o = _orthogonal_update(upd, g["ns_steps"])
                    upd = o * (rms / (o.pow(2).mean().sqrt() + 1e-12))
                if g["weight_decay"]:
                    p.mul_(1 - g["lr"] * g["weight_decay"])
                p.add_(upd.to(p.dtype), alpha=-g["lr"])
        return loss


def build_musgd_parameter_groups(model: torch.nn.Module, lr: float, weight_decay: float = 0.0,
                                 head_lr_scale: float = 1.0) -> List[dict]:
    body, head, nodecay = [], [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if "lm_head" in name or "embed" in name:
            head.append(p)
        elif p.ndim < 2:
            nodecay.append(p)
        else:
            body.append(p)
    groups = []
    if body:
        groups.append({"params": body, "lr": lr, "weight_decay": weight_decay, "name": "body"})
    if head:
        groups.append({"params": head, "lr": lr * head_lr_scale, "weight_decay": 0.0,
                       "name": "head"})
    if nodecay:
        groups.append({"params": nodecay, "lr": lr, "weight_decay": 0.0, "name": "vectors"})
    return groups


def named_learning_rates(optimizer: Optimizer) -> Dict[str, float]:
    return {g.get("name", f"group{i}"): float(g["lr"]) for i, g in enumerate(optimizer.param_groups)}


# ------------------------------------------------------------ other families
class Lion(Optimizer):
    """Lion (Chen et al., 2023): sign of an interpolated momentum."""

    def __init__(self, params, lr: float = 1e-4, betas=(0.9, 0.99), weight_decay: float = 0.0):
        super().__init__(params, dict(lr=lr, betas=betas, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            b1, b2 = g["betas"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                grad = p.grad.float()
                st = self.state[p]
                if not st:
                    st["exp_avg"] = torch.zeros_like(grad)
                m = st["exp_avg"]
                upd = (m * b1 + grad * (1 - b1)).sign_()
                if g["weight_decay"]:
                    p.mul_(1 - g["lr"] * g["weight_decay"])
                p.add_(upd.to(p.dtype), alpha=-g["lr"])
                m.mul_(b2).add_(grad, alpha=1 - b2)
        return loss


class Sophia(Optimizer):
    """Sophia-G (Liu et al., 2023): momentum preconditioned by an EMA of a
    diagonal Gauss-Newton estimate, element-wise clipped to [-1, 1].

    Call :meth:`update_hessian` every ``k`` steps after a backward pass of the
    loss on labels sampled from the model (the Gauss-Newton-Bartlett
    estimator): it folds ``grad**2 * batch_size`` into the estimate.
    """

    def __init__(self, params, lr: float = 1e-4, betas=(0.965, 0.99), rho: float = 0.04,
                 weight_decay: float = 0.1, eps: float = 1e-15):
        super().__init__(params, dict(lr=lr, betas=betas, rho=rho, weight_decay=weight_decay,
                                      eps=eps))

    @torch.no_grad()
    def update_hessian(self, batch_size: int = 1) -> None:
        for g in self.param_groups:
            b2 = g["betas"][1]
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self._init(p)
                st["hessian"].mul_(b2).addcmul_(p.grad.float(), p.grad.float(),
                                                value=(1 - b2) * batch_size)

    def _init(self, p):
        st = self.state[p]
        if not st:
            st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
            st["hessian"] = torch.zeros_like(p, dtype=torch.float32)
        return st

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None, bs: int = 1):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            b1 = g["betas"][0]
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self._init(p)
                st["exp_avg"].mul_(b1).add_(p.grad.float(), alpha=1 - b1)
                if g["weight_decay"]:
                    p.mul_(1 - g["lr"] * g["weight_decay"])
                ratio = (st["exp_avg"].abs() / (g["rho"] * bs * st["hessian"] + g["eps"])).clamp(
                    max=1.0)
                p.add_((st["exp_avg"].sign() * ratio).to(p.dtype), alpha=-g["lr"])
        return loss


_Q_BLOCK = 256


def _quantize_signed(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Blockwise absmax int8 quantisation of a flat fp32 tensor."""
    n = x.numel()
    pad = (-n) % _Q_BLOCK
    xb = torch.nn.functional.pad(x.reshape(-1), (0, pad)).view(-1, _Q_BLOCK)
    scale = xb.abs().amax(dim=1).clamp_min(1e-12)
    q = torch.round(xb / scale[:, None] * 127).to(torch.int8)
    return q, scale


def _dequantize_signed(q: torch.Tensor, scale: torch.Tensor, n: int) -> torch.Tensor:
    return (q.float() * (scale[:, None] / 127)).reshape(-1)[:n]


def _quantize_unsigned_sqrt(v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Second moments are stored as sqrt(v) in uint8 blocks (halves the dynamic range)."""
    s = v.reshape(-1).clamp_min(0).sqrt()
    n = s.numel()
    pad = (-n) % _Q_BLOCK
    sb = torch.nn.functional.pad(s, (0, pad)).view(-1, _Q_BLOCK)
    scale = sb.amax(dim=1).clamp_min(1e-20)
    q = torch.round(sb / scale[:, None] * 255).to(torch.uint8)
    return q, scale


def _dequantize_unsigned_sqrt(q, scale, n):
    return ((q.float() * (scale[:, None] / 255)).reshape(-1)[:n]).square()


class Adam8bit(Optimizer):
    """AdamW with block-wise 8-bit optimizer state (256-element blocks, absmax
    scales): first moment int8, second moment stored as sqrt in uint8.
    Tensors smaller than ``min_8bit_size`` keep fp32 state."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, min_8bit_size: int = 4096):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                      min_8bit_size=min_8bit_size))

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            b1, b2 = g["betas"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                grad = p.grad.float().reshape(-1)
                n = grad.numel()
                st = self.state[p]
                q8 = n >= g["min_8bit_size"]
                if not st:
                    st["step"] = 0
                    if q8:
                        st["m_q"], st["m_s"] = _quantize_signed(torch.zeros_like(grad))
                        st["v_q"], st["v_s"] = _quantize_unsigned_sqrt(torch.zeros_like(grad))
                    else:
                        st["exp_avg"] = torch.zeros_like(grad)
                        st["exp_avg_sq"] = torch.zeros_like(grad)
                st["step"] += 1
                if q8:
                    m = _dequantize_signed(st["m_q"], st["m_s"], n)
                    v = _dequantize_unsigned_sqrt(st["v_q"], st["v_s"], n)
                else:
                    m, v = st["exp_avg"], st["exp_avg_sq"]
                m.lerp_(grad, 1 - b1)
                v.mul_(b2).addcmul_(grad, grad, value=1 - b2)
                upd = (m / (1 - b1 ** st["step"])) / ((v / (1 - b2 ** st["step"])).sqrt() + g["eps"])
                if q8:
                    st["m_q"], st["m_s"] = _quantize_signed(m)
                    st["v_q"], st["v_s"] = _quantize_unsigned_sqrt(v)
                if g["weight_decay"]:
                    p.mul_(1 - g["lr"] * g["weight_decay"])
                p.add_(upd.view_as(p).to(p.dtype), alpha=-g["lr"])
        return loss


def _factored_rms(row: torch.Tensor, col: torch.Tensor) -> torch.Tensor:
    """Rank-1 reconstruction of a second moment from its row/column means."""
    r = row / row.mean(dim=-1, keepdim=True).clamp_min(1e-30)
    return torch.rsqrt(r.unsqueeze(-1) * col.unsqueeze(-2))


class CAME(Optimizer):
    """CAME (Luo et al., 2023): Adafactor-style factored second moments plus a
    factored confidence term from the instability (update - momentum)^2."""

    def __init__(self, params, lr: float = 2e-4, betas=(0.9, 0.999, 0.9999),
                 eps=(1e-30, 1e-16), clip_threshold: float = 1.0, weight_decay: float = 0.0):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps,
                                      clip_threshold=clip_threshold, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            b1, b2, b3 = g["betas"]
            e1, e2 = g["eps"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                grad = p.grad.float()
                st = self.state[p]
                factored = grad.ndim >= 2
                if not st:
                    st["exp_avg"] = torch.zeros_like(grad)
                    if factored:
                        st["row"] = torch.zeros(grad.shape[:-1], device=grad.device)
                        st["col"] = torch.zeros(grad.shape[:-2] + grad.shape[-1:], device=grad.device)
                        st["res_row"] = torch.zeros_like(st["row"])
                        st["res_col"] = torch.zeros_like(st["col"])
                    else:
                        st["exp_avg_sq"] = torch.zeros_like(grad)
                g2 = grad.square() + e1
                if factored:
                    st["row"].mul_(b2).add_(g2.mean(dim=-1), alpha=1 - b2)
                    st["col"].mul_(b2).add_(g2.mean(dim=-2), alpha=1 - b2)
                    upd = grad * _factored_rms(st["row"], st["col"])
                else:
                    st["exp_avg_sq"].mul_(b2).add_(g2, alpha=1 - b2)
                    upd = grad * st["exp_avg_sq"].rsqrt()
                rms = upd.pow(2).mean().sqrt()
                upd = upd / (rms / g["clip_threshold"]).clamp_min(1.0)
                m = st["exp_avg"]
                m.mul_(b1).add_(upd, alpha=1 - b1)
                if factored:
                    res = (upd - m).square() + e2
                    st["res_row"].mul_(b3).add_(res.mean(dim=-1), alpha=1 - b3)
                    st["res_col"].mul_(b3).add_(res.mean(dim=-2), alpha=1 - b3)
                    final = m * _factored_rms(st["res_row"], st["res_col"])
                else:
                    final = m
                if g["weight_decay"]:
                    p.mul_(1 - g["lr"] * g["weight_decay"])
                p.add_(final.to(p.dtype), alpha=-g["lr"])
        return loss


class AdaLomo(Optimizer):
    """AdaLomo (Lv et al., 2023): momentum-free factored second moments with
    grouped update normalisation (update RMS clipped to ``clip_threshold``
    and scaled by max(eps, RMS(param)))."""

    def __init__(self, params, lr: float = 1e-3, beta: float = 0.999, eps=(1e-30, 1e-3),
                 clip_threshold: float = 1.0, weight_decay: float = 0.0):
        super().__init__(params, dict(lr=lr, beta=beta, eps=eps, clip_threshold=clip_threshold,
                                      weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure: Optional[Callable] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for g in self.param_groups:
            e1, e2 = g["eps"]
            b = g["beta"]
            for p in g["params"]:
                if p.grad is None:
                    continue
                grad = p.grad.float()
                st = self.state[p]
                factored = grad.ndim >= 2
                if not st:
                    if factored:
                        st["row"] = torch.zeros(grad.shape[:-1], device=grad.device)
                        st["col"] = torch.zeros(grad.shape[:-2] + grad.shape[-1:], device=grad.device)
                    else:
                        st["v"] = torch.zeros_like(grad)
                g2 = grad.square() + e1
                if factored:
                    st["row"].mul_(b).add_(g2.mean(dim=-1), alpha=1 - b)
                    st["col"].mul_(b).add_(g2.mean(dim=-2), alpha=1 - b)
                    upd = grad * _factored_rms(st["row"], st["col"])
                else:
                    st["v"].mul_(b).add_(g2, alpha=1 - b)
                    upd = grad * st["v"].rsqrt()
                upd = upd / (upd.pow(2).mean().sqrt() / g["clip_threshold"]).clamp_min(1.0)
                scale = max(e2, float(p.detach().float().pow(2).mean().sqrt()))
                if g["weight_decay"]:
                    p.mul_(1 - g["lr"] * g["weight_decay"])
                p.add_(upd.to(p.dtype), alpha=-g["lr"] * scale)
        return loss


# ------------------------------------------------------------------- factory
def _decay_groups(model: torch.nn.Module, weight_decay: float) -> List[dict]:
    decay, nodecay = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if "bias" in name or "norm" in name or "embed" in name:
            nodecay.append(p)
        else:
            decay.append(p)
    return [{"params": decay, "weight_decay": weight_decay},
            {"params": nodecay, "weight_decay": 0.0}]


OPTIMIZER_NAMES = ("adamw", "adam", "sgd", "lion", "sophia", "adam8bit", "came", "adalomo", "muon",
                   "muon_tr", "adam_tr", "musgd")


def get_optimizer(model: torch.nn.Module, optimizer_type: str = "adamw", lr: float = 1e-4,
                  weight_decay: float = 0.01, **kwargs) -> Optimizer:
    """Build an optimizer by name (the LR conventions of the reference factory:
    Lion lr/10, Sophia lr/2, AdaLomo lr*10)."""
    kind = optimizer_type.lower()
    num_experts = int(kwargs.pop("num_experts", 4))
    if kind == "muon":
        mg, ag = split_params_for_muon(model)
        return MuonWithAdamW(mg, ag, lr=kwargs.pop("muon_lr", 0.02), adam_lr=lr,
                             weight_decay=weight_decay, **kwargs)
    if kind == "muon_tr":
        return MuonTR(tr_param_groups(model, num_experts, weight_decay=weight_decay),
                      lr=kwargs.pop("muon_lr", 0.003), adam_lr=lr, num_experts=num_experts,
                      **kwargs)
    if kind == "adam_tr":
        return AdamTR(tr_param_groups(model, num_experts, weight_decay=weight_decay), lr=lr,
                      num_experts=num_experts, weight_decay=weight_decay, **kwargs)
    groups = _decay_groups(model, weight_decay)
    table = {
        "adamw": lambda: torch.optim.AdamW(groups, lr=lr, **kwargs),
        "adam": lambda: torch.optim.Adam(groups, lr=lr, **kwargs),
        "sgd": lambda: torch.optim.SGD(groups, lr=lr, **kwargs),
        "lion": lambda: Lion(groups, lr=lr / 10, **kwargs),
        "sophia": lambda: Sophia(groups, lr=lr / 2, **kwargs),
        "adam8bit": lambda: Adam8bit(groups, lr=lr, **kwargs),
        "came": lambda: CAME(groups, lr=lr, **kwargs),
        "adalomo": lambda: AdaLomo(groups, lr=lr * 10, **kwargs),
        "musgd": lambda: MuSGD(build_musgd_parameter_groups(model, lr, weight_decay), lr=lr,
                               **kwargs),
    }
    if kind not in table:
        raise ValueError(f"unknown optimizer {optimizer_type!r}; available: {list(OPTIMIZER_NAMES)}")
    return table[kind]()


class DistributedOptimizer:
    """Wraps any ``torch.optim.Optimizer`` with the Trainer's step protocol:
    ``reduce_gradients`` (one all-reduce per flattened bucket, averaged),
    ``clip_grad_norm_`` and ``step(clip=...)``."""

    def __init__(self, optimizer: Optimizer, process_group=None, bucket_bytes: int = 64 << 20):
        self.optimizer = optimizer
        self.pg = process_group
        self.bucket_bytes = bucket_bytes
        on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(process_group) if on else 1

    @property
    def param_groups(self):
        return self.optimizer.param_groups

    @property
    def state(self):
        return self.optimizer.state

    def _params(self) -> List[torch.nn.Parameter]:
        return [p for g in self.optimizer.param_groups for p in g["params"]]

    @torch.no_grad()
    def reduce_gradients(self) -> None:
        if self.world == 1:
            return
        grads = [p.grad for p in self._params() if p.grad is not None]
        bucket, size = [], 0
        for gr in grads + [None]:
            if gr is not None:
                bucket.append(gr)
                size += gr.numel() * gr.element_size()
            if bucket and (gr is None or size >= self.bucket_bytes):
                flat = torch.cat([b.reshape(-1).float() for b in bucket])
                dist.all_reduce(flat, group=self.pg)
                flat /= self.world
                off = 0
                for b in bucket:
                    b.copy_(flat[off:off + b.numel()].view_as(b))
                    off += b.numel()
                bucket, size = [], 0

    def clip_grad_norm_(self, max_norm: float) -> torch.Tensor:
        return torch.nn.utils.clip_grad_norm_(self._params(), max_norm)

    def step(self, closure=None, clip: bool = False):
        return self.optimizer.step(closure)

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.optimizer.zero_grad(set_to_none=set_to_none)

    def state_dict(self) -> Dict:
        return self.optimizer.state_dict()

    def load_state_dict(self, sd: Dict) -> None:
        self.optimizer.load_state_dict(sd)
