"""Megatron-style tensor parallelism for the TR-Hash decoder.

Shards, over a TP group of size P:
  * attention: q heads (and k/v heads when divisible by P, else replicated),
    o_proj input columns;
  * the shared SwiGLU: gate/up output rows, down input columns;
  * every routed expert: its width W (gate/up columns, down rows);
so one decoder block needs exactly one all-reduce after attention and one
after the FFN.  The reference shards attention only and leaves the FFN
replicated (complexity/parallel/tensor_parallel.py:371-446), and
its backward never all-reduces the gradient of the replicated input
(``_AllReduceFunc`` backward is identity with no copy-to-region op); here ``copy_to_tp`` (identity forward, all-reduce backward) and
``reduce_from_tp`` (all-reduce forward, identity backward) pair up correctly.

The primitives and ``ColumnParallelLinear`` / ``RowParallelLinear`` /
``ParallelEmbedding`` keep the reference names.  Each sharded parameter
records ``_tp_shard_dim`` so checkpoints can be re-assembled
(``gather_tp_state_dict``).
"""
from __future__ import annotations

from dataclasses import replace
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

_TP = {"group": None}


def initialize_tensor_parallel(group) -> None:
    _TP["group"] = group


def get_tp_group():
    return _TP["group"]


def tp_world(group=None) -> int:
    g = group if group is not None else _TP["group"]
    return dist.get_world_size(g) if (g is not None and dist.is_initialized()) else 1


def tp_rank(group=None) -> int:
    g = group if group is not None else _TP["group"]
    return dist.get_rank(g) if (g is not None and dist.is_initialized()) else 0


# ------------------------------------------------------------- primitives
class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherLastDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        P = dist.get_world_size(group)
        parts = [torch.empty_like(x) for _ in range(P)]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, -1)

    @staticmethod
    def backward(ctx, g):
        P = dist.get_world_size(ctx.group)
        r = dist.get_rank(ctx.group)
        return g.chunk(P, -1)[r].contiguous(), None


class _ScatterLastDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        P = dist.get_world_size(group)
        return x.chunk(P, -1)[dist.get_rank(group)].contiguous()

    @staticmethod
    def backward(ctx, g):
        P = dist.get_world_size(ctx.group)
        parts = [torch.empty_like(g) for _ in range(P)]
        dist.all_gather(parts, g.contiguous(), group=ctx.group)
        return torch.cat(parts, -1), None


def copy_to_tp(x, group=None):
    g = group if group is not None else _TP["group"]
    return x if tp_world(g) == 1 else _CopyToTP.apply(x, g)


def reduce_from_tp(x, group=None):
    g = group if group is not None else _TP["group"]
    return x if tp_world(g) == 1 else _ReduceFromTP.apply(x, g)


def gather_from_tp(x, group=None):
    g = group if group is not None else _TP["group"]
    return x if tp_world(g) == 1 else _GatherLastDim.apply(x, g)


def scatter_to_tp(x, group=None):
    g = group if group is not None else _TP["group"]
    return x if tp_world(g) == 1 else _ScatterLastDim.apply(x, g)


# ------------------------------------------------------------------ layers
class ColumnParallelLinear(nn.Module):
    """y = x W^T with W split by output rows; optional gather of the output."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 gather_output: bool = False, group=None):
        super().__init__()
        self.group = group if group is not None else _TP["group"]
        P = tp_world(self.group)
        if out_features % P:
            raise ValueError("out_features must be divisible by the TP size")
        self.gather_output = gather_output
        self.weight = nn.Parameter(torch.empty(out_features // P, in_features))
        self.weight._tp_shard_dim = 0
        self.bias = nn.Parameter(torch.zeros(out_features // P)) if bias else None
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, x):
        y = F.linear(copy_to_tp(x, self.group), self.weight, self.bias)
        return gather_from_tp(y, self.group) if self.gather_output else y


class RowParallelLinear(nn.Module):
    """y = sum_ranks x_r W_r^T with W split by input columns (all-reduce of the output)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 input_is_parallel: bool = True, group=None):
        super().__init__()
        self.group = group if group is not None else _TP["group"]
        P = tp_world(self.group)
        if in_features % P:
            raise ValueError("in_features must be divisible by the TP size")
        self.input_is_parallel = input_is_parallel
        self.weight = nn.Parameter(torch.empty(out_features, in_features // P))
        self.weight._tp_shard_dim = 1
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, x):
        if not self.input_is_parallel:
            x = scatter_to_tp(x, self.group)
        y = reduce_from_tp(F.linear(x, self.weight), self.group)
        return y + self.bias if self.bias is not None else y


class ParallelEmbedding(nn.Module):
    """Vocabulary-sharded embedding: each rank owns V/P rows; outputs are all-reduced."""

    def __init__(self, num_embeddings: int, embedding_dim: int, group=None):
        super().__init__()
        self.group = group if group is not None else _TP["group"]
        P, r = tp_world(self.group), tp_rank(self.group)
        if num_embeddings % P:
            raise ValueError("vocab must be divisible by the TP size")
        self.per = num_embeddings // P
        self.lo = r * self.per
        self.weight = nn.Parameter(torch.empty(self.per, embedding_dim))
        self.weight._tp_shard_dim = 0
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, ids):
        local = ids - self.lo
        mask = (local < 0) | (local >= self.per)
        out = F.embedding(local.clamp(0, self.per - 1), self.weight)
        out = out.masked_fill(mask[..., None], 0.0)
        return reduce_from_tp(out, self.group)


# ------------------------------------------------------------- model surgery
def _shard(p: torch.Tensor, dim: int, P: int, r: int) -> nn.Parameter:
    n = p.shape[dim]
    if n % P:
        raise ValueError(f"dimension {dim} of size {n} is not divisible by TP size {P}")
    out = nn.Parameter(p.detach().narrow(dim, r * (n // P), n // P).clone(),
                       requires_grad=p.requires_grad)
    out._tp_shard_dim = dim
    return out


def _block_split(n: int, P: int, r: int, block: int):
    """(start, size) of rank r's share of n columns dealt in whole blocks:
    the first (n/block) % P ranks get one block more."""
    nb = n // block
    per, extra = divmod(nb, P)
    start = (r * per + min(r, extra)) * block
    return start, (per + (1 if r < extra else 0)) * block


def _shard_range(p: torch.Tensor, dim: int, start: int, size: int, sizes) -> nn.Parameter:
    out = nn.Parameter(p.detach().narrow(dim, start, size).clone(), requires_grad=p.requires_grad)
    out._tp_shard_dim = dim
    out._tp_shard_sizes = tuple(sizes)
    return out


def make_parallel(model: nn.Module, group=None, shared_block: int = 0) -> nn.Module:
    """Shard a full-weight ``ComplexityModel`` in place over ``group`` (default: TP group).

    Load the full checkpoint first; each rank keeps its slice.  Embedding and
    LM head stay replicated (their gradients are averaged by data parallelism
    or are identical across TP ranks).  With ``shared_block`` > 0 a shared
    SwiGLU width whose even split is not a multiple of the block is dealt in
    whole blocks instead (ranks may then hold different widths, e.g. 11008 over
    8 ranks as 11 or 10 blocks of 128), which keeps every rank on the fused
    SwiGLU kernel.
    """
    group = group if group is not None else _TP["group"]
    P, r = tp_world(group), tp_rank(group)
    if P == 1:
        return model
    initialize_tensor_parallel(group)
    for layer in model.layers:
        a = layer.self_attn
        if a.num_heads % P:
            raise ValueError("num_attention_heads must be divisible by the TP size")
        D = a.head_dim
        a.q_proj.weight = _shard(a.q_proj.weight, 0, P, r)
        if a.num_kv_heads % P == 0:
            a.k_proj.weight = _shard(a.k_proj.weight, 0, P, r)
            a.v_proj.weight = _shard(a.v_proj.weight, 0, P, r)
            a.num_kv_heads //= P
        else:
            # keep every KV head; this rank's q heads use the kv heads they map to
            keep = a.num_kv_heads
            per_q = a.num_heads // P
            groups = a.num_heads // keep
            first_kv = (r * per_q) // groups
            last_kv = ((r + 1) * per_q - 1) // groups
            n_kv = last_kv - first_kv + 1
            if per_q % n_kv:
                raise ValueError("KV heads cannot be assigned evenly to the TP ranks")
            sl = slice(first_kv * D, (last_kv + 1) * D)
            for name in ("k_proj", "v_proj"):
                lin = getattr(a, name)
                lin.weight = nn.Parameter(lin.weight.detach()[sl].clone())
                lin.weight._tp_replicated_kv = True
            a.num_kv_heads = n_kv
        a.num_heads //= P
        a.num_kv_groups = a.num_heads // a.num_kv_heads
        a.o_proj.weight = _shard(a.o_proj.weight, 1, P, r)
        a.tp_group = group
        eng = getattr(layer.mlp, "engine", None)
        if eng is not None:
            cfg = eng.config
            sw = cfg.shared_width
            blocked = (shared_block > 0 and sw % shared_block == 0
                       and (sw % P or (sw // P) % shared_block))
            if cfg.expert_width % P or (sw % P and not blocked):
                raise ValueError("expert and shared widths must be divisible by the TP size")
            local_sw = sw // P
            if eng.shared_gate is not None:
                if blocked:
                    sizes = [_block_split(sw, P, q, shared_block)[1] for q in range(P)]
                    start, local_sw = _block_split(sw, P, r, shared_block)
                    eng.shared_gate.weight = _shard_range(eng.shared_gate.weight, 0, start,
                                                          local_sw, sizes)
                    eng.shared_up.weight = _shard_range(eng.shared_up.weight, 0, start,
                                                        local_sw, sizes)
                    eng.shared_down.weight = _shard_range(eng.shared_down.weight, 1, start,
                                                          local_sw, sizes)
                else:
                    eng.shared_gate.weight = _shard(eng.shared_gate.weight, 0, P, r)
                    eng.shared_up.weight = _shard(eng.shared_up.weight, 0, P, r)
                    eng.shared_down.weight = _shard(eng.shared_down.weight, 1, P, r)
            eng.expert_gate = _shard(eng.expert_gate, 2, P, r)
            eng.expert_up = _shard(eng.expert_up, 2, P, r)
            eng.expert_down = _shard(eng.expert_down, 1, P, r)
            eng.config = replace(cfg, shared_width=local_sw,
                                 expert_width=cfg.expert_width // P)
            eng._active_expert_width = eng.config.expert_width
            eng.tp_group = group
    model.tp_group = group
    return model


def gather_tp_state_dict(model: nn.Module, group=None) -> dict:
    """Full (unsharded) state dict from a TP-sharded model (collective over the TP group)."""
    group = group if group is not None else getattr(model, "tp_group", _TP["group"])
    P = tp_world(group)
    shard_dims, shard_sizes = {}, {}
    for name, p in model.named_parameters():
        if hasattr(p, "_tp_shard_dim"):
            shard_dims[name] = p._tp_shard_dim
            shard_sizes[name] = getattr(p, "_tp_shard_sizes", None)
    out = {}
    for name, t in model.state_dict().items():
        if name in shard_dims and P > 1:
            dim, sizes = shard_dims[name], shard_sizes[name]
            if sizes is None:
                parts = [torch.empty_like(t) for _ in range(P)]
                dist.all_gather(parts, t.contiguous(), group=group)
                t = torch.cat(parts, dim)
            else:  # uneven block shards: gather padded to the largest, then trim
                big = max(sizes)
                pad = list(t.shape)
                pad[dim] = big
                buf = t.new_zeros(pad)
                buf.narrow(dim, 0, t.shape[dim]).copy_(t)
                parts = [torch.empty_like(buf) for _ in range(P)]
                dist.all_gather(parts, buf, group=group)
                t = torch.cat([q.narrow(dim, 0, n) for q, n in zip(parts, sizes)], dim)
        out[name] = t
    return out


# --------------------------------------------------- reference helper names
# complexity/parallel/tensor_parallel.py:29-175 keeps the TP group in module
# state built from an integer size; the same calls work here on top of the
# group-based primitives above.
def init_tensor_parallel_group(tp_size) -> None:
    """Create the TP groups (consecutive ranks, ``tp_size`` each; every rank must
    call) and make this rank's group the default; a process group may be passed
    instead of a size."""
    if not (dist.is_available() and dist.is_initialized()):
        _TP["group"] = None
        return
    if not isinstance(tp_size, int):
        _TP["group"] = tp_size
        return
    world = dist.get_world_size()
    if tp_size <= 1:
        _TP["group"] = None
        return
    if world % tp_size:
        raise ValueError(f"world size {world} is not divisible by tp_size {tp_size}")
    mine = None
    for start in range(0, world, tp_size):
        g = dist.new_group(list(range(start, start + tp_size)))
        if start <= dist.get_rank() < start + tp_size:
            mine = g
    _TP["group"] = mine


def get_tensor_parallel_world_size() -> int:
    return tp_world()


def get_tensor_parallel_rank() -> int:
    return tp_rank()


def get_tensor_parallel_group():
    return _TP["group"]


def all_reduce(tensor: torch.Tensor) -> torch.Tensor:
    """Sum over the TP group (identity gradient)."""
    return reduce_from_tp(tensor)


class _ReduceScatterDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, group):
        ctx.dim, ctx.group = dim, group
        parts = [p.contiguous() for p in x.chunk(dist.get_world_size(group), dim)]
        out = torch.empty_like(parts[0])
        dist.reduce_scatter(out, parts, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        parts = [torch.empty_like(g) for _ in range(dist.get_world_size(ctx.group))]
        dist.all_gather(parts, g.contiguous(), group=ctx.group)
        return torch.cat(parts, ctx.dim), None, None


class _AllGatherDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, group):
        ctx.dim, ctx.group = dim, group
        parts = [torch.empty_like(x) for _ in range(dist.get_world_size(group))]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim)

    @staticmethod
    def backward(ctx, g):
        P = dist.get_world_size(ctx.group)
        parts = [p.contiguous() for p in g.chunk(P, ctx.dim)]
        out = torch.empty_like(parts[0])
        dist.reduce_scatter(out, parts, group=ctx.group)
        return out, None, None


def reduce_scatter(tensor: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Sum over the TP group, keep this rank's slice along ``dim`` (backward: all-gather)."""
    g = _TP["group"]
    return tensor if tp_world(g) == 1 else _ReduceScatterDim.apply(tensor, dim, g)


def all_gather(tensor: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Concatenate every rank's tensor along ``dim`` (backward: reduce-scatter)."""
    g = _TP["group"]
    return tensor if tp_world(g) == 1 else _AllGatherDim.apply(tensor, dim, g)
