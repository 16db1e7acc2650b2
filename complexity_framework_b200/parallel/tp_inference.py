"""Tensor-parallel paged decoding: sharded weights, one fused all-reduce per
attention and per FFN, CUDA-graph friendly.

``enable_tp_decode(model, group)`` shards a full-weight ``ComplexityModel``
over the ranks of ``group`` (``make_parallel``: local query/KV heads, o_proj
input columns, the shared SwiGLU and every expert split along their width;
the shared width goes in 128-column blocks so every rank stays on the fused
SwiGLU kernel even when the width does not divide evenly), then attaches a
``TPDecodeComm``.  In eval mode each layer ends attention and the FFN with a
partial written straight into a symmetric buffer, and ``C.tp_allreduce``
(csrc/tp_decode.cu) returns ``residual + sum of partials`` in one launch: a
bounded device barrier over the signal pads, then every rank reads all
partials over NVLink (or one ``multimem.ld_reduce`` through the NVSwitch when
the buffer has a multicast address).  Epochs live on the device, so a decode
step captured in a CUDA graph replays with fresh barriers.

Rows beyond ``max_rows`` (long prefill chunks) use an NCCL all-reduce.
Embedding and LM head stay replicated, so every rank computes the same logits
and the engines on all ranks stay in lockstep without extra traffic.

Reference counterpart: ``make_parallel`` + the TP linear layers of
complexity/parallel/tensor_parallel.py:371-438 (attention-only sharding,
NCCL all-reduce per row-parallel linear).
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch
import torch.distributed as dist


class TPDecodeComm:
    """Per-call-site symmetric partial buffers, signal pads and device epoch of
    one tensor-parallel group."""

    def __init__(self, group, hidden: int, n_sites: int, max_rows: int = 256,
                 device: Optional[torch.device] = None, multicast: Optional[bool] = None):
        import torch.distributed._symmetric_memory as symm

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if not 1 <= self.world <= 8:
            raise ValueError("decode tensor parallelism supports 1..8 ranks in one node")
        self.device = torch.device(device or "cuda", torch.cuda.current_device())
        self.hidden, self.n_sites, self.max_rows = hidden, n_sites, max_rows
        self.site_elems = max_rows * hidden
        pad = symm.empty(4 * 8, dtype=torch.int32, device=self.device)
        pad.zero_()
        hp = symm.rendezvous(pad, self.group)
        buf = symm.empty(n_sites * self.site_elems, dtype=torch.bfloat16, device=self.device)
        buf.zero_()
        hb = symm.rendezvous(buf, self.group)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._keep = (pad, hp, buf, hb)
        self.pads = self._peer_ptrs(hp, pad)
        self.bufs = self._peer_ptrs(hb, buf)
        self.buf = buf
        want_mc = (os.environ.get("CFB_TP_NVLS", "1") != "0") if multicast is None else multicast
        mc = int(getattr(hb, "multicast_ptr", 0) or 0) if want_mc else 0
        self.mc = mc + (buf.data_ptr() - int(hb.buffer_ptrs[hb.rank])) if mc else 0
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=self.device)

    @staticmethod
    def _peer_ptrs(h, t) -> List[int]:
        off = t.data_ptr() - int(h.buffer_ptrs[h.rank])
        return [int(p) + off for p in h.buffer_ptrs]

    @property
    def uses_multicast(self) -> bool:
        return self.mc != 0

    def fits(self, rows: int) -> bool:
        return rows <= self.max_rows

    def partial(self, site: int, rows: int) -> torch.Tensor:
        """This rank's buffer for call site ``site``: write the partial here."""
        base = site * self.site_elems
        return self.buf[base:base + rows * self.hidden].view(rows, self.hidden)

    def allreduce(self, site: int, rows: int, residual: Optional[torch.Tensor]) -> torch.Tensor:
        """``residual + sum over ranks`` of the partials written at ``site``."""
        from ..ops import require

        n = rows * self.hidden
        off = site * self.site_elems * 2  # bytes
        out = torch.empty(rows, self.hidden, device=self.device, dtype=torch.bfloat16)
        r = None if residual is None else residual.reshape(rows, self.hidden).contiguous()
        require().tp_allreduce([b + off for b in self.bufs], self.pads,
                               self.mc + off if self.mc else 0, self.rank, r, out.view(-1)[:n],
                               self.epoch, self.ticket)
        return out


def tp_reduce_add(comm: Optional[TPDecodeComm], site: int, partial_fn, rows: int,
                  residual: Optional[torch.Tensor], group) -> torch.Tensor:
    """``residual + all-reduce(partial)``: the fused kernel when the rows fit the
    site buffers, else an NCCL all-reduce.  ``partial_fn(out)`` writes the
    partial into ``out`` (a [rows, H] bf16 tensor) and returns it."""
    if comm is not None and comm.fits(rows):
        partial_fn(comm.partial(site, rows))
        return comm.allreduce(site, rows, residual)
    part = partial_fn(None)
    part = part.contiguous().clone()
    dist.all_reduce(part, group=group)
    return part if residual is None else residual.reshape(part.shape) + part


def enable_tp_decode(model, group=None, max_rows: int = 256, multicast: Optional[bool] = None):
    """Shard ``model`` for tensor-parallel decoding over ``group`` and attach the
    fused all-reduce.  Returns the model (sharded in place)."""
    from .tensor_parallel import make_parallel

    group = group if group is not None else dist.group.WORLD
    make_parallel(model, group, shared_block=128)
    dev = next(model.parameters()).device
    if dist.get_world_size(group) == 1 or dev.type != "cuda":
        return model  # CPU: the per-layer all-reduces go through the process group
    comm = TPDecodeComm(group, model.config.hidden_size, 2 * len(model.layers), max_rows,
                        multicast=multicast)
    for i, layer in enumerate(model.layers):
        layer.self_attn.tp_decode = comm
        layer.self_attn.tp_site = 2 * i
        eng = getattr(layer.mlp, "engine", None)
        if eng is not None:
            eng.tp_decode = comm
            eng.tp_site = 2 * i + 1
    model.tp_decode = comm
    return model
