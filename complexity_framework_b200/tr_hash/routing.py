"""Deterministic token-ID route tables.

A route table is a CPU int64 tensor ``[top_k, vocab_size]``: entry ``[j, t]``
is the expert of token id ``t`` in route slot ``j``.  Fresh models regenerate
the tables from the config, so every builder must be bit-exact with the
reference (complexity/tr_hash/routing.py:12-259): the seeds, the 32-bit hash
``mix32`` (a murmur-style finaliser), the use of ``torch.Generator`` /
``torch.randperm`` and ``topk`` tie-breaking are part of the checkpoint
contract and are therefore kept identical.  The code below is written from
the algorithm description; all arithmetic is int64 masked to 32 bits.
"""
from __future__ import annotations

from dataclasses import replace

import torch

from .config import TRHashEngineConfig, TRHashStrategy

_M32 = 0xFFFFFFFF
_LAYER_PRIME = 104729
_GOLDEN = 0x9E3779B1
_C1 = 0x85EBCA77
_C2 = 0xC2B2AE3D


def mix32(x: torch.Tensor) -> torch.Tensor:
    """32-bit avalanche hash of an int64 tensor (values kept in [0, 2^32))."""
    x = x & _M32
    for shift, mult in ((16, 0x7FEB352D), (15, 0x846CA68B)):
        x = (x ^ (x >> shift)) & _M32
        x = (x * mult) & _M32
    return (x ^ (x >> 16)) & _M32


def _randperm(n: int, seed: int) -> torch.Tensor:
    gen = torch.Generator(device="cpu").manual_seed(int(seed))
    return torch.randperm(n, generator=gen, device="cpu")


def _layer_permutation(num_experts: int, layer_index: int, seed: int) -> torch.Tensor:
    return _randperm(num_experts, int(seed) + _LAYER_PRIME * int(layer_index))


def _layer_salt(cfg: TRHashEngineConfig) -> int:
    return (int(cfg.route_seed) + int(cfg.layer_index) * _GOLDEN) & _M32


def modulo_cyclic_routes(cfg: TRHashEngineConfig) -> torch.Tensor:
    perm = _layer_permutation(cfg.num_experts, cfg.layer_index, cfg.route_seed ^ 0xC0DE)
    primary = perm[torch.arange(cfg.vocab_size, dtype=torch.long) % cfg.num_experts]
    slots = [(primary + j) % cfg.num_experts for j in range(cfg.top_k)]
    return torch.stack(slots, 0)


def balanced_hash_routes(cfg: TRHashEngineConfig) -> torch.Tensor:
    """Each block of ``E`` consecutive ranks uses every expert once per slot."""
    E, V = cfg.num_experts, cfg.vocab_size
    if E == 1:
        return torch.zeros(cfg.top_k, V, dtype=torch.long)
    order = _randperm(V, int(cfg.route_seed) + _LAYER_PRIME * int(cfg.layer_index))
    rank = torch.arange(V, dtype=torch.long)
    block, offset = rank // E, rank % E
    odd = torch.arange(1, E, 2, dtype=torch.long)
    pick = mix32(block + int(cfg.route_seed) + int(cfg.layer_index) * _GOLDEN) % odd.numel()
    stride = odd[pick]
    perm = _layer_permutation(E, cfg.layer_index, cfg.route_seed ^ 0x5EC0D)
    by_rank = torch.stack([perm[(offset + j * stride) % E] for j in range(cfg.top_k)], 0)
    routes = torch.empty(cfg.top_k, V, dtype=torch.long)
    routes[:, order] = by_rank
    return routes


def affine_hash_routes(cfg: TRHashEngineConfig) -> torch.Tensor:
    t = torch.arange(cfg.vocab_size, dtype=torch.int64)
    salt = _layer_salt(cfg)
    base = mix32(t ^ salt) % cfg.num_experts
    stride = (mix32(t + (salt ^ _C1)) | 1) % cfg.num_experts
    return torch.stack([(base + j * stride) % cfg.num_experts for j in range(cfg.top_k)], 0).long()


def multi_hash_routes(cfg: TRHashEngineConfig) -> torch.Tensor:
    """Rendezvous voting: the top-k experts by a sum of per-channel hashes."""
    t = torch.arange(cfg.vocab_size, dtype=torch.int64)[:, None]
    e = torch.arange(cfg.num_experts, dtype=torch.int64)[None, :]
    salt = _layer_salt(cfg)
    score = torch.zeros(cfg.vocab_size, cfg.num_experts, dtype=torch.int64)
    for h in range(cfg.route_hash_count):
        ch = (salt + h * _C1) & _M32
        score += mix32(t ^ mix32(e + (ch ^ _C2)) ^ ch)
    return score.topk(cfg.top_k, dim=1, largest=True, sorted=True).indices.T.long()


def expand_route_table_hierarchically(routes: torch.Tensor, *, source_num_experts: int,
                                      target_num_experts: int, layer_index: int,
                                      route_seed: int = 0x71D5A17) -> torch.Tensor:
    """Replace each parent expert ``p`` by one of its clones ``p + c*source``."""
    if routes.ndim != 2:
        raise ValueError("routes must be shaped [top_k, vocab_size]")
    if source_num_experts < 1:
        raise ValueError("source_num_experts must be positive")
    if target_num_experts <= source_num_experts:
        raise ValueError("target_num_experts must exceed source_num_experts")
    if target_num_experts % source_num_experts:
        raise ValueError("target_num_experts must be a multiple of source_num_experts")
    if routes.numel() and (int(routes.min()) < 0 or int(routes.max()) >= source_num_experts):
        raise ValueError("routes contain an invalid source expert index")
    clones = target_num_experts // source_num_experts
    t = torch.arange(routes.size(1), dtype=torch.int64)[None, :]
    slot = torch.arange(routes.size(0), dtype=torch.int64)[:, None]
    parent = routes.detach().to("cpu", torch.int64)
    salt = (int(route_seed) + int(layer_index) * _GOLDEN) & _M32
    clone = mix32(t ^ (parent * _C1) ^ (slot * _C2) ^ salt) % clones
    return (parent + clone * source_num_experts).long()


def hierarchical_hash_routes(cfg: TRHashEngineConfig) -> torch.Tensor:
    if cfg.num_experts < 4 or cfg.num_experts % 2:
        raise ValueError("hierarchical hash requires an even expert count of at least four")
    parents = cfg.num_experts // 2
    if cfg.top_k > parents:
        raise ValueError("top_k cannot exceed the hierarchical parent expert count")
    parent_cfg = replace(cfg, num_experts=parents, routing_strategy=TRHashStrategy.BALANCED_HASH)
    return expand_route_table_hierarchically(
        balanced_hash_routes(parent_cfg), source_num_experts=parents,
        target_num_experts=cfg.num_experts, layer_index=cfg.layer_index,
        route_seed=cfg.route_seed)


_BUILDERS = {
    TRHashStrategy.BALANCED_HASH: balanced_hash_routes,
    TRHashStrategy.MODULO_CYCLIC: modulo_cyclic_routes,
    TRHashStrategy.AFFINE_HASH: affine_hash_routes,
    TRHashStrategy.MULTI_HASH: multi_hash_routes,
    TRHashStrategy.HIERARCHICAL_HASH: hierarchical_hash_routes,
}


def build_route_table(config: TRHashEngineConfig) -> torch.Tensor:
    """CPU ``[top_k, vocab_size]`` int64 route table, validated.

    Always built on the CPU, also under a meta / CUDA default-device context
    (e.g. deferred initialisation by model loaders)."""
    with torch.device("cpu"):
        routes = _BUILDERS[config.routing_strategy](config)
    if tuple(routes.shape) != (config.top_k, config.vocab_size):
        raise RuntimeError("route builder returned an invalid shape")
    with torch.device("cpu"):
        if int(routes.min()) < 0 or int(routes.max()) >= config.num_experts:
            raise RuntimeError("route builder returned an invalid expert index")
        if config.top_k > 1:
            s = routes.sort(dim=0).values
            if bool((s[1:] == s[:-1]).any()):
                raise RuntimeError("route builder selected one expert twice")
    return routes


# ------------------------------------------------------------ top-2 pair codes
def _pair_layout(pair_count: int):
    """(index mask, swap bit) of the one-byte pair code."""
    return (0x7, 0x8) if pair_count <= 8 else (0x1F, 0x20)


def compile_top2_pair_metadata(routes: torch.Tensor, *, num_experts: int):
    """Encode a top-2 table as ``uint8[vocab]`` codes plus an ``int32[P,2]`` pair list.

    The pair list is ``torch.combinations(arange(E), 2)``; a code is the index of
    the unordered pair, with the swap bit set when slot 0 holds the larger id.
    """
    if routes.ndim != 2 or routes.size(0) != 2:
        raise ValueError("routes must be shaped [2, vocab_size]")
    if not 2 <= num_experts <= 8:
        raise ValueError("compact pair metadata supports two to eight experts")
    if routes.numel() and (int(routes.min()) < 0 or int(routes.max()) >= num_experts):
        raise ValueError("routes contain an invalid expert index")
    pairs = torch.combinations(torch.arange(num_experts, dtype=torch.int32), r=2)
    P = int(pairs.size(0))
    if P > 32:
        raise ValueError("compact pair encoding supports at most 32 pairs")
    r = routes.detach().to("cpu", torch.long)
    lo, hi = r.min(dim=0).values, r.max(dim=0).values
    if bool((lo == hi).any()):
        raise ValueError("top-2 pair routes must select two distinct experts")
    # index of the unordered pair (lo, hi) in lexicographic combinations order
    lookup = torch.full((num_experts, num_experts), -1, dtype=torch.long)
    lookup[pairs[:, 0].long(), pairs[:, 1].long()] = torch.arange(P)
    idx = lookup[lo, hi]
    if bool((idx < 0).any()):
        raise ValueError("routes contain an expert pair that cannot be encoded")
    _, swap_bit = _pair_layout(P)
    swap = (r[0] == hi).long()
    codes = (idx | (swap * swap_bit)).to(torch.uint8)
    return codes, pairs


def decode_top2_pair_metadata(route_codes: torch.Tensor, expert_pairs: torch.Tensor) -> torch.Tensor:
    if route_codes.ndim != 1 or route_codes.dtype != torch.uint8:
        raise ValueError("route_codes must be a one-dimensional uint8 tensor")
    if expert_pairs.ndim != 2 or expert_pairs.size(1) != 2:
        raise ValueError("expert_pairs must be shaped [pair_count, 2]")
    P = int(expert_pairs.size(0))
    mask, swap_bit = _pair_layout(P)
    codes = route_codes.to(torch.int64)
    idx = codes & mask
    if idx.numel() and int(idx.max()) >= P:
        raise ValueError("route_codes reference an unavailable expert pair")
    sel = expert_pairs[idx].long()
    swap = (codes & swap_bit) != 0
    first = torch.where(swap, sel[:, 1], sel[:, 0])
    second = torch.where(swap, sel[:, 0], sel[:, 1])
    return torch.stack((first, second), 0)
