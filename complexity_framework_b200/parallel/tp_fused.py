"""Tensor parallelism with the collectives fused into the GEMMs (sequence parallel).

Activations between tensor-parallel regions are sharded by token rows: rank p
holds rows [p*T/P, (p+1)*T/P) of the flattened [T, H] stream.

* ``ag_linear`` (column parallel): Y[T, N/P] = AllGather(X)[T, H] @ W_p^T in ONE
  GEMM kernel.  Two copier warps of every CTA pull the peers' 128-row chunks
  over NVLink (each remote byte crosses once) into this rank's gathered buffer
  and publish per-chunk flags; the TMA producer computes this rank's own row
  tiles first and waits (bounded) for a chunk's flag before loading its rows,
  so the transfer overlaps the tensor-core work tile by tile.  The gathered
  buffer stays valid for the backward weight gradient.
* ``rs_linear`` (row parallel): Out_p = sum_q (X_q @ W_q^T)[rows of p] (+ R_p).
  The GEMM stores its bf16 partial into this rank's symmetric buffer; the
  finish kernel announces completion, waits (bounded) for every peer and sums
  the owned rows of all partials (peer rows by 16-byte NVLink loads, read once)
  with the residual in fp32.
* Backward: d(ag_linear) is a reduce-scatter of dY @ W_p; d(rs_linear) is an
  all-gather GEMM of dOut with W_p; weight gradients read the gathered buffers.

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
        self.flag_bufs: Dict[str, torch.Tensor] = {}
        self.flag_uses: Dict[str, int] = {}
        self.views: Dict[str, torch.Tensor] = {}

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
        view = t[:n].view(*shape)
        self.views[name] = view
        return view, ptrs

    def flags(self, name: str, n: int):
        """Local int32 chunk counters of call site ``name`` and the number of uses
        including this one (a chunk is complete when its counter reaches
        uses x pieces-per-chunk; counters are never reset)."""
        f = self.flag_bufs.get(name)
        if f is None or f.numel() < n:
            f = torch.zeros(n, dtype=torch.int32, device=self.device)
            self.flag_bufs[name] = f
            self.flag_uses[name] = 0
        self.flag_uses[name] += 1
        return f[:n], self.flag_uses[name]

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
    """``AllGather(x_shard) @ op(w)`` with the gather inside the GEMM: copier warps
    pull the peers' row chunks (once each) into this rank's gathered buffer while
    the tensor cores work on this rank's own rows."""
    C = require()
    rows, K = x_shard.shape
    T = rows * ws.world
    g, ptrs = ws.buffer(name, (T, K), torch.bfloat16)
    g[ws.rank * rows:(ws.rank + 1) * rows].copy_(x_shard)
    flags, uses = ws.flags(name, T // 128)
    N = w.shape[1] if b_mn else w.shape[0]
    e = ws.epoch(ROUND_AG)
    tail = (ws.pads, ws.rank, ROUND_AG, e, 0, True, ptrs, flags, rows, uses)
    if epi == EPI_SWIGLU_FWD:
        C.gemm_dist(g, False, w, b_mn, T, N, K, epi, None, epi_kw["gu"], epi_kw["act"],
                    epi_kw.get("row_scale"), epi_kw["shared_width"], epi_kw["expert_width"],
                    epi_kw["n_experts"], epi_kw["shared_scale"], [], 0, [], 0, [], 0, *tail)
        return epi_kw["act"]
    out = epi_kw.get("out")
    if out is None:
        out = torch.empty(T, N, device=x_shard.device, dtype=torch.bfloat16)
    C.gemm_dist(g, False, w, b_mn, T, N, K, epi, out, epi_kw.get("gu"), None,
                epi_kw.get("row_scale"), epi_kw.get("shared_width", 0),
                epi_kw.get("expert_width", 1), epi_kw.get("n_experts", 0),
                epi_kw.get("shared_scale", 1.0), [], 0, [], 0, [], 0, *tail)
    return out


def gathered(ws: TPWorkspace, name: str) -> torch.Tensor:
    """This rank's complete gathered buffer of call site ``name`` (after its AG GEMM)."""
    return ws.views[name]


def _rs_gemm(ws: TPWorkspace, name: str, a: torch.Tensor, w: torch.Tensor, b_mn: bool,
             residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Reduce-scatter of ``a @ op(w)`` by rows: returns this rank's [T/P, N] rows.

    The GEMM writes its bf16 partial of all rows into this rank's symmetric
    buffer (TMA stores); the finish kernel reads the peers' partials of the
    rows this rank owns over NVLink, once, and sums them with its own.
    """
    C = require()
    T, K = a.shape
    N = w.shape[1] if b_mn else w.shape[0]
    rows = _shard_rows(T, ws.world)
    part, ptrs = ws.buffer(name, (T, N), torch.bfloat16)
    C.gemm(a, False, w, b_mn, T, N, K, EPI_STORE, out=part)
    out = torch.empty(rows, N, device=a.device, dtype=torch.bfloat16)
    C.tp_rs_finish(ptrs, rows, N, N, residual, out, ws.pads, ws.rank, ROUND_RS,
                   ws.epoch(ROUND_RS))
    return out


def _wgrad_gathered_b(ws: TPWorkspace, name: str, dy: torch.Tensor, n_rows: int, K: int
                      ) -> torch.Tensor:
    """dW = dY^T @ AllGather(X), reading the gathered X that the forward GEMM left
    in this rank's buffer ``name`` (no second transfer)."""
    from ..ops.fused import gemm_tn

    return gemm_tn(dy, gathered(ws, name), out_dtype=torch.float32)


def _wgrad_gathered_a(ws: TPWorkspace, name: str, x_local: torch.Tensor, n_out: int
                      ) -> torch.Tensor:
    """dW = AllGather(dOut)^T @ X_local, with the gathered dOut left in buffer ``name``."""
    from ..ops.fused import gemm_tn

    return gemm_tn(gathered(ws, name), x_local, out_dtype=torch.float32)


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


class TPMLPFn(torch.autograd.Function):
    """TR-Hash MLP under fused sequence-parallel TP: gate|up all-gather GEMM with
    the SwiGLU + route-scale epilogue, down projection as a reduce-scatter GEMM
    with the residual added in the finish kernel.  Backward: the down data
    gradient is an all-gather GEMM with the SwiGLU-backward epilogue."""

    @staticmethod
    def forward(ctx, h_shard, w_gu, w_down, row_scale, residual, ws, name, sw, ew, ne, ss):
        rows, H = h_shard.shape
        T = rows * ws.world
        A2 = w_gu.shape[0]
        dev = h_shard.device
        gu = torch.empty(T, A2, device=dev, dtype=torch.bfloat16)
        act = torch.empty(T, A2 // 2, device=dev, dtype=torch.bfloat16)
        _ag_gemm(ws, name + ".h", h_shard.contiguous(), w_gu.contiguous(), False, EPI_SWIGLU_FWD,
                 gu=gu, act=act, row_scale=row_scale, shared_width=sw, expert_width=ew,
                 n_experts=ne, shared_scale=ss)
        out = _rs_gemm(ws, name + ".down", act, w_down.contiguous(), False,
                       residual.contiguous() if residual is not None else None)
        ctx.save_for_backward(w_gu, w_down, row_scale, gu, act)
        ctx.meta = (ws, name, sw, ew, ne, ss, residual is not None)
        return out

    @staticmethod
    def backward(ctx, dout):
        w_gu, w_down, row_scale, gu, act = ctx.saved_tensors
        ws, name, sw, ew, ne, ss, has_res = ctx.meta
        from ..ops.fused import gemm_tn

        T, A2 = gu.shape
        dgu = torch.empty(T, A2, device=gu.device, dtype=torch.bfloat16)
        _ag_gemm(ws, name + ".dy", dout.contiguous(), w_down, True, EPI_SWIGLU_BWD, out=dgu, gu=gu,
                 row_scale=row_scale, shared_width=sw, expert_width=ew, n_experts=ne,
                 shared_scale=ss)
        dw_down = gemm_tn(gathered(ws, name + ".dy"), act).to(w_down.dtype)
        dh = _rs_gemm(ws, name + ".dh", dgu, w_gu, True)
        dw_gu = gemm_tn(dgu, gathered(ws, name + ".h")).to(w_gu.dtype)
        return (dh, dw_gu, dw_down, None, dout if has_res else None, None, None, None, None, None,
                None)


def enable_fused_sequence_parallel(model, group=None):
    """Shard ``model`` for tensor parallelism (heads, shared and expert widths)
    and switch its CUDA forward to the fused sequence-parallel path."""
    from .tensor_parallel import make_parallel, tp_world

    group = group if group is not None else dist.group.WORLD
    if tp_world(group) < 2:
        raise ValueError("fused sequence parallelism needs a group of 2..8 ranks")
    make_parallel(model, group)
    ws = TPWorkspace(group)
    model.sp_ws = ws
    for layer in model.layers:
        if getattr(layer.self_attn, "num_kv_heads", 1) and any(
                getattr(p, "_tp_replicated_kv", False) for p in layer.self_attn.parameters()):
            raise ValueError("fused sequence parallelism needs KV heads divisible by the TP size")
    return model


def replicated_parameters(model):
    """Parameters every TP rank holds in full (embeddings, norms, LM head): their
    gradients are partial per rank under sequence parallelism."""
    return [p for p in model.parameters() if p.requires_grad and not hasattr(p, "_tp_shard_dim")]


def allreduce_replicated_grads(model, group=None) -> None:
    grads = [p.grad for p in replicated_parameters(model) if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1).float() for g in grads])
    dist.all_reduce(flat, group=group or model.sp_ws.group)
    off = 0
    for g in grads:
        g.copy_(flat[off:off + g.numel()].view_as(g))
        off += g.numel()
