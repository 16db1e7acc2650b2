"""Tensor parallelism with the collectives fused into the GEMMs (sequence parallel).

Activations between tensor-parallel regions are sharded by token rows: rank p
holds rows [p*T/P, (p+1)*T/P) of the flattened [T, H] stream.  The two
collectives of a Megatron-style layer are fused into the sm_100a GEMM:

* ``ag_linear`` (column parallel): Y[T, N/P] = AllGather(X)[T, H] @ W_p^T.
  Each rank's X shard lives in symmetric memory; the GEMM's TMA producer loads
  the A tiles of rows owned by rank q straight from q's buffer over NVLink
  (one tensor map per rank, plain TMA loads, never multicast), after a bounded
  device barrier that confirms every shard is written.  Backward: dX is a
  reduce-scatter GEMM (below) of dY @ W_p; dW_p = dY^T @ AllGather(X) reads
  the peers' X shards again through segmented TMA loads.
* ``rs_linear`` (row parallel): Out_p = sum_q (X_q @ W_q^T)[rows of p] (+ R_p).
  The GEMM epilogue stores each fp32 partial tile straight into the owning
  rank's slot for this source rank (NVLink stores); a finish kernel announces
  completion, waits (bounded) for every peer and sums the slots of its own
  rows (+ residual) into bf16.  Backward: d(X_p) = AllGather(dOut) @ W_p (the
  gather fused into the loads again), dW_p = AllGather(dOut)^T @ X_p.

Reference counterpart: the (unfused) ``ColumnParallelLinear`` /
``RowParallelLinear`` of complexity/parallel/tensor_parallel.py:181-311, which
issue separate NCCL all-reduces.  Buffers are per call site (name), so a
shard stays readable by peers until the next step's forward; ``begin_step``
adds one device barrier per step so no rank rewrites a buffer a peer may still
read from the previous backward.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from ..ops._ext import require

EPI_STORE, EPI_SWIGLU_FWD, EPI_SWIGLU_BWD, EPI_F32_ATOMIC, EPI_PEER_STORE = 0, 2, 3, 7, 8
ROUND_AG, ROUND_RS, ROUND_STEP = 0, 1, 2


class TPWorkspace:
    """Symmetric buffers and signal pads of one tensor-parallel group."""

    def __init__(self, group=None, device=None):
        import torch.distributed._symmetric_memory as symm

        self.symm = symm
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if not 1 < self.world <= 8:
            raise ValueError("fused tensor parallelism supports 2..8 ranks in one node")
        self.device = torch.device(device or "cuda", torch.cuda.current_device())
        self.pad_buf, self.pads = self._alloc((4 * 8,), torch.int32, zero=True)
        self.epochs = [0, 0, 0, 0]
        self.buffers: Dict[str, Tuple[torch.Tensor, List[int]]] = {}

    def _alloc(self, shape, dtype, zero=False):
        n = 1
        for d in shape:
            n *= d
        t = self.symm.empty(n, dtype=dtype, device=self.device)
        if zero:
            t.zero_()
        h = self.symm.rendezvous(t, self.group)
        off = t.data_ptr() - h.buffer_ptrs[h.rank]
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        return t.view(*shape), [int(p) + off for p in h.buffer_ptrs]

    def buffer(self, name: str, shape, dtype) -> Tuple[torch.Tensor, List[int]]:
        """Per-call-site symmetric buffer (allocated collectively on first use)."""
        n = 1
        for d in shape:
            n *= d
        cur = self.buffers.get(name)
        if cur is None or cur[0].numel() < n or cur[0].dtype != dtype:
            self.buffers[name] = self._alloc((n,), dtype)
            cur = self.buffers[name]
        t, ptrs = cur
        return t[:n].view(*shape), ptrs

    def epoch(self, rnd: int) -> int:
        self.epochs[rnd] += 1
        return self.epochs[rnd]

    def begin_step(self) -> None:
        require().tp_barrier(self.pads, self.rank, ROUND_STEP, self.epoch(ROUND_STEP),
                             self.device.index)


def _shard_rows(T: int, world: int) -> int:
    if T % world or (T // world) % 128:
        raise ValueError(f"token rows {T} must split into {world} shards of a multiple of 128")
    return T // world


def _ag_gemm(ws: TPWorkspace, name: str, x_shard: torch.Tensor, w: torch.Tensor, b_mn: bool,
             epi: int = EPI_STORE, **epi_kw) -> torch.Tensor:
    """``AllGather(x_shard) @ op(w)`` with the gather fused into the GEMM loads."""
    C = require()
    rows, K = x_shard.shape
    T = rows * ws.world
    buf, ptrs = ws.buffer(name, (rows, K), torch.bfloat16)
    buf.copy_(x_shard)
    N = w.shape[1] if b_mn else w.shape[0]
    e = ws.epoch(ROUND_AG)
    if epi == EPI_SWIGLU_FWD:
        C.gemm_dist(buf, False, w, b_mn, T, N, K, epi, None, epi_kw["gu"], epi_kw["act"],
                    epi_kw.get("row_scale"), epi_kw["shared_width"], epi_kw["expert_width"],
                    epi_kw["n_experts"], epi_kw["shared_scale"], ptrs, rows, [], 0, [], 0,
                    ws.pads, ws.rank, ROUND_AG, e, 1, True)
        return epi_kw["act"]
    out = epi_kw.get("out")
    if out is None:
        out = torch.empty(T, N, device=x_shard.device, dtype=torch.bfloat16)
    C.gemm_dist(buf, False, w, b_mn, T, N, K, epi, out, epi_kw.get("gu"), None,
                epi_kw.get("row_scale"), epi_kw.get("shared_width", 0),
                epi_kw.get("expert_width", 1), epi_kw.get("n_experts", 0),
                epi_kw.get("shared_scale", 1.0), ptrs, rows, [], 0, [], 0, ws.pads, ws.rank,
                ROUND_AG, e, 1, True)
    return out


def _rs_gemm(ws: TPWorkspace, name: str, a: torch.Tensor, w: torch.Tensor, b_mn: bool,
             residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Reduce-scatter of ``a @ op(w)`` by rows: returns this rank's [T/P, N] rows."""
    C = require()
    T, K = a.shape
    N = w.shape[1] if b_mn else w.shape[0]
    rows = _shard_rows(T, ws.world)
    slots, ptrs = ws.buffer(name, (ws.world * rows, N), torch.float32)
    C.gemm_dist(a, False, w, b_mn, T, N, K, EPI_PEER_STORE, slots, None, None, None, 0, 1, 0,
                1.0, [], 0, [], 0, ptrs, rows, ws.pads, ws.rank, ROUND_RS, 0, 0, False)
    out = torch.empty(rows, N, device=a.device, dtype=torch.bfloat16)
    C.tp_rs_finish(slots, ws.world, rows, N, residual, out, ws.pads, ws.rank, ROUND_RS,
                   ws.epoch(ROUND_RS))
    return out


def _wgrad_gathered_b(ws: TPWorkspace, name: str, dy: torch.Tensor, n_rows: int, K: int
                      ) -> torch.Tensor:
    """dW = dY^T @ AllGather(X) where X's shards sit in buffer ``name`` (MN-major B
    segmented along the token dimension)."""
    C = require()
    T, N = dy.shape
    buf, ptrs = ws.buffers[name]
    rows = T // ws.world
    out = torch.zeros(N, K, device=dy.device, dtype=torch.float32)
    C.gemm_dist(dy, True, buf[:rows * K].view(rows, K), True, N, K, T, EPI_F32_ATOMIC, out, None,
                None, None, 0, 1, 0, 1.0, [], 0, ptrs, rows, [], 0, [], 0, 0, 0, 0, False)
    return out


def _wgrad_gathered_a(ws: TPWorkspace, name: str, x_local: torch.Tensor, n_out: int
                      ) -> torch.Tensor:
    """dW = AllGather(dOut)^T @ X_local where dOut's shards sit in buffer ``name``
    (MN-major A segmented along the token dimension)."""
    C = require()
    T, K = x_local.shape
    buf, ptrs = ws.buffers[name]
    rows = T // ws.world
    out = torch.zeros(n_out, K, device=x_local.device, dtype=torch.float32)
    C.gemm_dist(buf[:rows * n_out].view(rows, n_out), True, x_local, True, n_out, K, T,
                EPI_F32_ATOMIC, out, None, None, None, 0, 1, 0, 1.0, ptrs, rows, [], 0, [], 0,
                [], 0, 0, 0, 0, False)
    return out


class AGLinearFn(torch.autograd.Function):
    """Column-parallel linear on a token-sharded input: [T/P, K] -> [T, N_p]."""

    @staticmethod
    def forward(ctx, x_shard, w, ws, name):
        y = _ag_gemm(ws, name + ".x", x_shard.contiguous(), w.contiguous(), False)
        ctx.save_for_backward(w)
        ctx.ws, ctx.name, ctx.K = ws, name, x_shard.shape[1]
        return y

    @staticmethod
    def backward(ctx, dy):
        (w,) = ctx.saved_tensors
        ws = ctx.ws
        dy = dy.contiguous()
        dx = _rs_gemm(ws, ctx.name + ".rs", dy, w, True)
        dw = _wgrad_gathered_b(ws, ctx.name + ".x", dy, w.shape[0], ctx.K).to(w.dtype)
        return dx, dw, None, None


class RSLinearFn(torch.autograd.Function):
    """Row-parallel linear to a token-sharded output: [T, K_p] -> [T/P, N] (+ residual)."""

    @staticmethod
    def forward(ctx, x, w, residual, ws, name):
        x = x.contiguous()
        out = _rs_gemm(ws, name + ".rs", x, w.contiguous(),
                       False, residual.contiguous() if residual is not None else None)
        ctx.save_for_backward(x, w)
        ctx.ws, ctx.name, ctx.has_res = ws, name, residual is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        x, w = ctx.saved_tensors
        ws = ctx.ws
        dout = dout.contiguous()
        dx = _ag_gemm(ws, ctx.name + ".dy", dout, w, True)
        dw = _wgrad_gathered_a(ws, ctx.name + ".dy", x, w.shape[0]).to(w.dtype)
        return dx, dw, (dout if ctx.has_res else None), None, None


def ag_linear(x_shard, w, ws: TPWorkspace, name: str):
    return AGLinearFn.apply(x_shard, w, ws, name)


def rs_linear(x, w, residual, ws: TPWorkspace, name: str):
    return RSLinearFn.apply(x, w, residual, ws, name)
