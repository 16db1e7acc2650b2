"""Autograd operators over the sm_100a kernels.

Every operator here runs only on CUDA bf16 tensors and calls the compiled
extension; callers choose between these and the eager reference math (CPU,
fp32, or ``use_custom_kernels=False``).  GEMM conventions are those of
``gemm_tc.cu``: ``C[M,N] = sum_k A(m,k) B(n,k)`` with each operand either
K-major or MN-major, so the data and weight gradients of ``y = x W^T`` need no
transposed copies:

    forward  y  = x  @ W^T   : A = x  (K-major)  B = W  (K-major)
    dgrad    dx = dy @ W     : A = dy (K-major)  B = W  (MN-major)
    wgrad    dW = dy^T @ x   : A = dy (MN-major) B = x  (MN-major)
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from ._ext import require

EPI_STORE, EPI_RESID, EPI_SWIGLU_FWD, EPI_SWIGLU_BWD, EPI_F32, EPI_F32_ACC, EPI_CE_STATS = range(7)
EPI_F32_ATOMIC = 7

_PAIR_UNITS = 74  # resident CTA pairs on a 148-SM B200


def _few_tiles(M: int, N: int) -> bool:
    """True when an M x N output has under two waves of 256x256 pair tiles."""
    return ((M + 255) // 256) * ((N + 255) // 256) < 2 * _PAIR_UNITS


_SKINNY = os.environ.get("CFB_SKINNY_GEMM", "1") != "0"


def _skinny(M: int, N: int, K: int) -> bool:
    """Decode-shaped ``x @ W^T``: at most 128 rows and too few output tiles to
    occupy the GPU (under half a wave of 256-wide tiles), with enough K to
    split."""
    return _SKINNY and M <= 128 and (N + 255) // 256 < _PAIR_UNITS and K >= 512 and N % 8 == 0


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


# --------------------------------------------------------------------- GEMMs
def gemm_nt(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
            alpha: float = 1.0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``alpha * x @ w.T (+ residual)`` for 2-D bf16 ``x [M,K]``, ``w [N,K]``."""
    C = require()
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    if _skinny(M, N, K):
        # few rows (decoding): the weight is the long operand.  C^T = W x^T puts
        # N on the 128/256-row tile side and splits K over CTAs with fp32
        # atomics, so enough CTAs stream the weight to saturate HBM; one fused
        # elementwise pass then transposes, scales, adds the residual and casts.
        Mp = (M + 31) // 32 * 32  # the GEMM's N side is a multiple of 32
        xp = x if Mp == M else torch.nn.functional.pad(x, (0, 0, 0, Mp - M))
        acc = torch.zeros(N, Mp, device=x.device, dtype=torch.float32)
        C.gemm(w, False, xp, False, N, Mp, K, EPI_F32_ATOMIC, out=acc)
        C.skinny_finish(acc, None if residual is None else _c(residual), out, alpha)
        return out
    if residual is not None:
        C.gemm(x, False, w, False, M, N, K, EPI_RESID, out=out, residual=_c(residual), alpha=alpha)
    else:
        C.gemm(x, False, w, False, M, N, K, EPI_STORE, out=out, alpha=alpha)
    return out


def gemm_nn(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``dy @ w`` for ``dy [M,N]``, ``w [N,K]`` (data gradient of a linear layer)."""
    C = require()
    M, N = dy.shape
    K = w.shape[1]
    out = torch.empty(M, K, device=dy.device, dtype=torch.bfloat16)
    C.gemm(dy, False, w, True, M, K, N, EPI_STORE, out=out)
    return out


def gemm_tn(dy: torch.Tensor, x: torch.Tensor, out_dtype=torch.bfloat16,
            accumulate_into: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``dy.T @ x`` for ``dy [T,N]``, ``x [T,K]`` (weight gradient of a linear layer)."""
    C = require()
    T, N = dy.shape
    K = x.shape[1]
    if accumulate_into is not None:
        C.gemm(dy, True, x, True, N, K, T, EPI_F32_ACC, out=accumulate_into)
        return accumulate_into
    if out_dtype == torch.float32 or _few_tiles(N, K):
        # split the token (K) dimension over CTAs and sum the slices with fp32 atomics
        out = torch.zeros(N, K, device=dy.device, dtype=torch.float32)
        C.gemm(dy, True, x, True, N, K, T, EPI_F32_ATOMIC, out=out)
        return out if out_dtype == torch.float32 else out.to(out_dtype)
    else:
        out = torch.empty(N, K, device=dy.device, dtype=torch.bfloat16)
        C.gemm(dy, True, x, True, N, K, T, EPI_STORE, out=out)
    return out


class LinearFn(torch.autograd.Function):
    """``y = x @ W^T (+ residual)`` on the tcgen05 GEMM."""

    @staticmethod
    def forward(ctx, x, w, residual):
        shape = x.shape
        x2 = _c(x.reshape(-1, shape[-1]))
        r2 = None if residual is None else residual.reshape(-1, w.shape[0])
        y = gemm_nt(x2, _c(w), r2)
        ctx.save_for_backward(x2, w)
        ctx.has_res = residual is not None
        ctx.shape = shape
        return y.view(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = _c(dy.reshape(-1, w.shape[0]))
        dx = gemm_nn(dy2, _c(w)).view(ctx.shape) if ctx.needs_input_grad[0] else None
        dw = gemm_tn(dy2, x2) if ctx.needs_input_grad[1] else None
        dr = dy if ctx.has_res else None
        return dx, dw, dr


def linear(x, w, residual=None):
    return LinearFn.apply(x, w, residual)


# ------------------------------------------------------------ TR-Hash MLP
def pack_gate_up(shared_gate: Optional[torch.Tensor], shared_up: Optional[torch.Tensor],
                 expert_gate: torch.Tensor, expert_up: torch.Tensor, block: int = 128):
    """Interleave gate and up rows in blocks of ``block`` for the SwiGLU epilogue.

    Row order of the result: gate[0:128], up[0:128], gate[128:256], up[128:256] ...
    where gate = [shared_gate ; expert_gate as (E*W, H)] and likewise up.
    """
    E, H, W = expert_gate.shape
    g_parts = [expert_gate.permute(0, 2, 1).reshape(E * W, H)]
    u_parts = [expert_up.permute(0, 2, 1).reshape(E * W, H)]
    if shared_gate is not None:
        g_parts.insert(0, shared_gate)
        u_parts.insert(0, shared_up)
    g = torch.cat(g_parts, 0) if len(g_parts) > 1 else g_parts[0]
    u = torch.cat(u_parts, 0) if len(u_parts) > 1 else u_parts[0]
    A = g.shape[0]
    nb = A // block
    return torch.stack((g.view(nb, block, H), u.view(nb, block, H)), 1).reshape(2 * A, H)


def pack_shared_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = 128) -> torch.Tensor:
    """Interleave gate/up rows in blocks of ``block`` (shared SwiGLU only, no experts)."""
    A, H = gate.shape
    nb = A // block
    return torch.stack((gate.view(nb, block, H), up.view(nb, block, H)), 1).reshape(2 * A, H)


def pack_down(shared_down: Optional[torch.Tensor], expert_down: torch.Tensor) -> torch.Tensor:
    """``[H, shared + E*W]`` down weight: shared columns then expert e's W columns."""
    E, W, H = expert_down.shape
    ed = expert_down.permute(2, 0, 1).reshape(H, E * W)
    return torch.cat((shared_down, ed), 1) if shared_down is not None else _c(ed)


_NO_SPLIT = 1 << 40  # row-index divisor meaning "no (outer, inner) split"


def _trhash_pack_geometry(As: int, E: int, H: int, W: int, block: int = 128):
    """Copy jobs packing (shared_gate, shared_up, expert_gate, expert_up,
    shared_down, expert_down) into (w_gu [2A, H], w_down [H, A]).

    Each job is ``(rows, cols, src(div, hi, lo, cs), dst offset, dst(div, hi, lo, cs))``
    in elements; see ``copy_jobs`` in csrc/pack.cu.  Gate index g lands on
    packed row ``(g // block) * 2 * block + g % block`` (+ block for up);
    expert e's column w of ``[E, H, W]`` is gate index ``As + e * W + w``.
    """
    A = As + E * W
    inter = (block, 2 * block * H, H, 1)
    e_off = (As // block) * 2 * block * H
    jobs = []
    if As:
        jobs.append(("sg", "gu", As, H, (_NO_SPLIT, 0, H, 1), 0, inter))
        jobs.append(("su", "gu", As, H, (_NO_SPLIT, 0, H, 1), block * H, inter))
    jobs.append(("eg", "gu", E * W, H, (W, H * W, 1, W), e_off, inter))
    jobs.append(("eu", "gu", E * W, H, (W, H * W, 1, W), e_off + block * H, inter))
    if As:
        jobs.append(("sd", "down", H, As, (_NO_SPLIT, 0, As, 1), 0, (_NO_SPLIT, 0, A, 1)))
    jobs.append(("ed", "down", H, E * W, (_NO_SPLIT, 0, 1, H), As, (_NO_SPLIT, 0, A, 1)))
    return jobs


def _run_jobs(jobs, tensors, reverse: bool):
    """Run pack (reverse=False: weights -> packed) or unpack (packed -> weights) jobs."""
    C = require()
    srcs, dsts, geom = [], [], []
    for name, packed, rows, cols, sg, off, pg in jobs:
        w = tensors[name].reshape(-1)
        pk = tensors[packed].reshape(-1)[off:]
        if reverse:
            srcs.append(pk)
            dsts.append(w)
            geom += [rows, cols, *pg, *sg]
        else:
            srcs.append(w)
            dsts.append(pk)
            geom += [rows, cols, *sg, *pg]
    C.copy_jobs(srcs, dsts, geom)


def pack_trhash_weights(sg, su, eg, eu, sd, ed, block: int = 128):
    """(w_gu [2A, H], w_down [H, A]) in one copy-jobs launch (no autograd)."""
    E, H, W = eg.shape
    As = 0 if sg is None else sg.shape[0]
    A = As + E * W
    dev = eg.device
    t = {"sg": sg, "su": su, "eg": _c(eg), "eu": _c(eu), "sd": sd, "ed": _c(ed),
         "gu": torch.empty(2 * A, H, device=dev, dtype=torch.bfloat16),
         "down": torch.empty(H, A, device=dev, dtype=torch.bfloat16)}
    if As:
        t.update(sg=_c(sg), su=_c(su), sd=_c(sd))
    _run_jobs(_trhash_pack_geometry(As, E, H, W, block), t, reverse=False)
    return t["gu"], t["down"]


class PackTRHashFn(torch.autograd.Function):
    """Differentiable ``pack_trhash_weights``: one launch each way."""

    @staticmethod
    def forward(ctx, sg, su, eg, eu, sd, ed):
        ctx.geom = (0 if sg is None else sg.shape[0], *eg.shape)
        return pack_trhash_weights(sg, su, eg, eu, sd, ed)

    @staticmethod
    def backward(ctx, d_gu, d_down):
        return _unpack_trhash_grads(ctx.geom, _c(d_gu), _c(d_down))


def _unpack_trhash_grads(geom, d_gu, d_down, down_transposed: bool = False):
    """(d shared_gate, d shared_up, d expert_gate, d expert_up, d shared_down,
    d expert_down) in bf16 from packed gradients (fp32 or bf16).  With
    ``down_transposed`` the down gradient arrives as ``[A, H]`` (its transpose)."""
    As, E, H, W = geom
    dev = d_gu.device
    bf = torch.bfloat16
    t = {"gu": d_gu, "down": d_down,
         "eg": torch.empty(E, H, W, device=dev, dtype=bf),
         "eu": torch.empty(E, H, W, device=dev, dtype=bf),
         "ed": torch.empty(E, W, H, device=dev, dtype=bf)}
    if As:
        t.update(sg=torch.empty(As, H, device=dev, dtype=bf),
                 su=torch.empty(As, H, device=dev, dtype=bf),
                 sd=torch.empty(H, As, device=dev, dtype=bf))
    jobs = _trhash_pack_geometry(As, E, H, W)
    if not down_transposed:
        _run_jobs(jobs, t, reverse=True)
    else:
        C = require()
        gu_jobs = [j for j in jobs if j[1] == "gu"]
        srcs, dsts, geo = [], [], []
        for name, packed, rows, cols, sg, off, pg in gu_jobs:
            srcs.append(d_gu.reshape(-1)[off:])
            dsts.append(t[name].reshape(-1))
            geo += [rows, cols, *pg, *sg]
        dT = d_down.reshape(-1)
        if As:  # sd[h, c] = dT[c, h]
            srcs.append(dT)
            dsts.append(t["sd"].reshape(-1))
            geo += [H, As, _NO_SPLIT, 0, 1, H, _NO_SPLIT, 0, As, 1]
        # ed[e, w, h] = dT[As + e * W + w, h]: plain rows
        srcs.append(dT[As * H:])
        dsts.append(t["ed"].reshape(-1))
        geo += [E * W, H, _NO_SPLIT, 0, H, 1, _NO_SPLIT, 0, H, 1]
        C.copy_jobs(srcs, dsts, geo)
    return t.get("sg"), t.get("su"), t["eg"], t["eu"], t.get("sd"), t["ed"]


def packable(sg, eg, block: int = 128) -> bool:
    """Whether the copy-jobs packing applies (shared width a multiple of ``block``;
    ``CFB_FUSED_PACK=0`` selects the torch packing ops instead)."""
    if os.environ.get("CFB_FUSED_PACK", "1") == "0":
        return False
    As = 0 if sg is None else sg.shape[0]
    E, H, W = eg.shape
    return As % block == 0 and (As + E * W) % block == 0


def _trhash_forward(ctx, h, w_gu, w_down, row_scale, residual, shared_width, expert_width,
                    n_experts, shared_scale):
    C = require()
    shape = h.shape
    h2 = _c(h.reshape(-1, shape[-1]))
    T, H = h2.shape
    A2 = w_gu.shape[0]
    A = A2 // 2
    gu = torch.empty(T, A2, device=h.device, dtype=torch.bfloat16)
    act = torch.empty(T, A, device=h.device, dtype=torch.bfloat16)
    C.gemm(h2, False, w_gu, False, T, A2, H, EPI_SWIGLU_FWD, gu=gu, act=act,
           row_scale=row_scale, shared_width=shared_width, expert_width=expert_width,
           n_experts=n_experts, shared_scale=shared_scale)
    Hout = w_down.shape[0]
    r2 = None if residual is None else residual.reshape(-1, Hout)
    out = gemm_nt(act, w_down, r2)
    ctx.save_for_backward(h2, w_gu, w_down, row_scale, gu, act)
    ctx.meta = (shared_width, expert_width, n_experts, shared_scale)
    ctx.has_res = residual is not None
    ctx.shape = shape
    return out.view(*shape[:-1], Hout)


def trhash_mlp_infer(h, w_gu, w_down, row_scale, shared_width, expert_width, n_experts,
                     shared_scale, out: Optional[torch.Tensor] = None,
                     residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Inference ``act @ Wd^T (+ residual)`` of ``TRHashMLPFn`` (no autograd state),
    written into ``out`` when given (e.g. a tensor-parallel partial buffer)."""
    C = require()
    H = h.shape[-1]
    h2 = _c(h.reshape(-1, H))
    T = h2.shape[0]
    A2 = w_gu.shape[0]
    act = torch.empty(T, A2 // 2, device=h.device, dtype=torch.bfloat16)
    if _skinny(T, A2, H):
        # few rows: swapped operands + split-K (see gemm_nt), SwiGLU in the pass
        # that transposes the fp32 result
        Tp = (T + 31) // 32 * 32
        hp = h2 if Tp == T else torch.nn.functional.pad(h2, (0, 0, 0, Tp - T))
        acc = torch.zeros(A2, Tp, device=h.device, dtype=torch.float32)
        C.gemm(w_gu, False, hp, False, A2, Tp, H, EPI_F32_ATOMIC, out=acc)
        C.skinny_swiglu(acc, _c(row_scale.float()), act, shared_width, expert_width, n_experts,
                        shared_scale)
    else:
        gu = torch.empty(T, A2, device=h.device, dtype=torch.bfloat16)
        C.gemm(h2, False, w_gu, False, T, A2, H, EPI_SWIGLU_FWD, gu=gu, act=act,
               row_scale=row_scale, shared_width=shared_width, expert_width=expert_width,
               n_experts=n_experts, shared_scale=shared_scale)
    r2 = None if residual is None else residual.reshape(T, w_down.shape[0])
    return gemm_nt(act, w_down, r2, out=out)


def _trhash_backward(ctx, dout, wgrad_dtype, down_transposed: bool = False):
    """(dh, dw_gu, dw_down, d residual); with ``down_transposed`` dw_down is
    returned as ``[A, Hout]``: the 3328 x 896 split-K product tiles better than
    its 896 x 3328 transpose."""
    C = require()
    h2, w_gu, w_down, row_scale, gu, act = ctx.saved_tensors
    sw, ew, ne, ss = ctx.meta
    T, H = h2.shape
    Hout, A = w_down.shape
    d2 = _c(dout.reshape(-1, Hout))
    dw_down = (gemm_tn(act, d2, out_dtype=wgrad_dtype) if down_transposed
               else gemm_tn(d2, act, out_dtype=wgrad_dtype))
    dgu = torch.empty(T, 2 * A, device=d2.device, dtype=torch.bfloat16)
    C.gemm(d2, False, w_down, True, T, A, Hout, EPI_SWIGLU_BWD, out=dgu, gu=gu,
           row_scale=row_scale, shared_width=sw, expert_width=ew, n_experts=ne,
           shared_scale=ss)
    dh = gemm_nn(dgu, w_gu).view(ctx.shape)
    dw_gu = gemm_tn(dgu, h2, out_dtype=wgrad_dtype)
    dr = dout if ctx.has_res else None
    return dh, dw_gu, dw_down, dr


class TRHashMLPFn(torch.autograd.Function):
    """Shared SwiGLU + deterministic routed experts (+ residual) as two GEMMs.

    act[:, c] = silu(g_c) * u_c * s(row, c), where s = shared_scale for shared
    columns and routed_scale * sum_j w_j [route_j(token) == expert(c)] for
    expert columns (zero when the token is not routed to that expert), then
    out = act @ Wd^T (+ residual).  Mathematically identical to
    reference_topk_swiglu (complexity/tr_hash/engine.py:66-104) with the shared
    branch of engine._shared (:333-349).
    """

    @staticmethod
    def forward(ctx, h, w_gu, w_down, row_scale, residual, shared_width, expert_width,
                n_experts, shared_scale):
        return _trhash_forward(ctx, h, _c(w_gu), _c(w_down), row_scale, residual, shared_width,
                               expert_width, n_experts, shared_scale)

    @staticmethod
    def backward(ctx, dout):
        dh, dw_gu, dw_down, dr = _trhash_backward(ctx, dout, torch.bfloat16)
        return dh, dw_gu, dw_down, None, dr, None, None, None, None


class TRHashMLPParamsFn(torch.autograd.Function):
    """``TRHashMLPFn`` over the unpacked parameters.

    The packed gate|up and down weights are built by one copy-jobs launch
    per forward, and the fp32 weight gradients (split-K atomics) are cast and
    scattered back to the six parameters by one launch in backward, instead of
    torch cat/stack/permute/cast kernels and their autograd inverses.
    """

    @staticmethod
    def forward(ctx, h, sg, su, eg, eu, sd, ed, row_scale, residual, shared_width,
                expert_width, n_experts, shared_scale):
        w_gu, w_down = pack_trhash_weights(sg, su, eg, eu, sd, ed)
        ctx.geom = (0 if sg is None else sg.shape[0], *eg.shape)
        return _trhash_forward(ctx, h, w_gu, w_down, row_scale, residual, shared_width,
                               expert_width, n_experts, shared_scale)

    @staticmethod
    def backward(ctx, dout):
        dh, dw_gu, dw_down, dr = _trhash_backward(ctx, dout, torch.float32, down_transposed=True)
        dsg, dsu, deg, deu, dsd, ded = _unpack_trhash_grads(ctx.geom, dw_gu, dw_down,
                                                            down_transposed=True)
        n = None
        return dh, dsg, dsu, deg, deu, dsd, ded, n, dr, n, n, n, n


def trhash_mlp(h, w_gu, w_down, row_scale, residual, shared_width, expert_width, n_experts,
               shared_scale):
    return TRHashMLPFn.apply(h, w_gu, w_down, row_scale, residual, shared_width, expert_width,
                             n_experts, shared_scale)


def trhash_mlp_params(h, sg, su, eg, eu, sd, ed, row_scale, residual, shared_width,
                      expert_width, n_experts, shared_scale):
    """TR-Hash MLP from the module's own parameters (shared ones may be None)."""
    return TRHashMLPParamsFn.apply(h, sg, su, eg, eu, sd, ed, row_scale, residual,
                                   shared_width, expert_width, n_experts, shared_scale)


def route_scales(token_ids: torch.Tensor, route_table: torch.Tensor, route_weights: torch.Tensor,
                 num_experts: int, routed_scale: float) -> torch.Tensor:
    C = require()
    ids = _c(token_ids.reshape(-1).long())
    out = torch.empty(ids.numel(), num_experts, device=ids.device, dtype=torch.float32)
    C.route_scales(ids, _c(route_table.long()), _c(route_weights.float()), out, num_experts,
                   float(routed_scale))
    return out


# ------------------------------------------------------------------ RMSNorm
def _norm_weight_grad(w: torch.Tensor, H: int) -> torch.Tensor:
    """Output buffer of d(norm weight): bf16, written directly by the kernel's
    last block, for H <= 1024; a zeroed fp32 accumulator otherwise."""
    if H <= 1024:
        return torch.empty(w.numel(), device=w.device, dtype=torch.bfloat16)
    return torch.zeros(w.numel(), device=w.device, dtype=torch.float32)


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        C = require()
        xc = _c(x)
        y = torch.empty_like(xc)
        H = x.shape[-1]
        rstd = torch.empty(xc.numel() // H, device=x.device, dtype=torch.float32)
        C.rmsnorm_fwd(xc, _c(w), y, rstd, float(eps))
        ctx.save_for_backward(xc, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        C = require()
        x, w, rstd = ctx.saved_tensors
        dx = torch.empty_like(x)
        dw = _norm_weight_grad(w, x.shape[-1])
        C.rmsnorm_bwd(_c(dy), x, _c(w), rstd, None, dx, dw)
        return dx, dw.to(w.dtype), None


def rmsnorm(x, w, eps):
    return RMSNormFn.apply(x, w, eps)


class RMSNormSkipFn(torch.autograd.Function):
    """``(rmsnorm(x), x)``: the second output is the residual stream itself.

    Routing the residual through the norm lets its backward receive both
    gradients of ``x`` (through the norm and through the skip connection) and
    sum them inside the RMSNorm-backward kernel instead of in a separate add.
    """

    @staticmethod
    def forward(ctx, x, w, eps):
        C = require()
        xc = _c(x)
        y = torch.empty_like(xc)
        H = x.shape[-1]
        rstd = torch.empty(xc.numel() // H, device=x.device, dtype=torch.float32)
        C.rmsnorm_fwd(xc, _c(w), y, rstd, float(eps))
        ctx.save_for_backward(xc, w, rstd)
        return y, x.view_as(x)

    @staticmethod
    def backward(ctx, dy, dskip):
        C = require()
        x, w, rstd = ctx.saved_tensors
        if dy is None:
            return dskip, None, None
        dx = torch.empty_like(x)
        dw = _norm_weight_grad(w, x.shape[-1])
        C.rmsnorm_bwd(_c(dy), x, _c(w), rstd, None if dskip is None else _c(dskip), dx, dw)
        return dx, dw.to(w.dtype), None


def rmsnorm_skip(x, w, eps):
    return RMSNormSkipFn.apply(x, w, eps)


# ---------------------------------------------------------- QK-norm + RoPE
class QKNormRopeFn(torch.autograd.Function):
    """kqv [B,S,(2Hkv+Hq)D] -> q [B,Hq,S,D], k/v [B,Hkv,S,D].

    k/v are head-major contiguous.  q is stored token-major ([B,S,Hq,D]
    memory, returned as its transposed view): SDPA then produces its output
    and dq token-major too, so the attention output feeds o_proj as a free
    ``[B,S,Hq*D]`` view instead of a per-layer transpose copy.
    """

    @staticmethod
    def forward(ctx, kqv, qw, kw, cos, sin, pos, Hq, Hkv, D, eps, qk_norm):
        C = require()
        B, S = kqv.shape[0], kqv.shape[1]
        kqv = _c(kqv)
        dev = kqv.device
        q = torch.empty(B, S, Hq, D, device=dev, dtype=torch.bfloat16)
        k = torch.empty(B, Hkv, S, D, device=dev, dtype=torch.bfloat16)
        v = torch.empty(B, Hkv, S, D, device=dev, dtype=torch.bfloat16)
        rstd = torch.empty(B * S, Hq + Hkv, device=dev, dtype=torch.float32)
        C.qk_norm_rope_fwd(kqv, _c(qw), _c(kw), cos, sin, pos, q, k, v, rstd, B, S, Hq, Hkv, D,
                           float(eps), bool(qk_norm), True)
        ctx.save_for_backward(kqv, qw, kw, cos, sin, rstd, pos)
        ctx.meta = (B, S, Hq, Hkv, D, bool(qk_norm))
        return q.transpose(1, 2), k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        C = require()
        kqv, qw, kw, cos, sin, rstd, pos = ctx.saved_tensors
        B, S, Hq, Hkv, D, qk_norm = ctx.meta
        dev = kqv.device
        dkqv = torch.empty_like(kqv)
        # bf16 weight gradients written by the kernel's last block (no fill / cast)
        dqw = torch.empty(D, device=dev, dtype=torch.bfloat16)
        dkw = torch.empty(D, device=dev, dtype=torch.bfloat16)

        def z(shape):
            return torch.zeros(shape, device=dev, dtype=torch.bfloat16)

        # token-major dq; SDPA already returns it in that layout (no copy)
        dq = dq.transpose(1, 2).contiguous() if dq is not None else z((B, S, Hq, D))
        dk = _c(dk) if dk is not None else z((B, Hkv, S, D))
        dv = _c(dv) if dv is not None else z((B, Hkv, S, D))
        C.qk_norm_rope_bwd(dq, dk, dv, kqv, _c(qw), _c(kw), cos, sin, pos, rstd, dkqv, dqw, dkw,
                           B, S, Hq, Hkv, D, qk_norm, True)
        n = None
        if not qk_norm:  # the weights are not used
            return (dkqv, n, n, n, n, n, n, n, n, n, n)
        return (dkqv, dqw.to(qw.dtype), dkw.to(kw.dtype), n, n, n, n, n, n, n, n)


def qk_norm_rope(kqv, qw, kw, cos, sin, pos, Hq, Hkv, D, eps, qk_norm=True):
    return QKNormRopeFn.apply(kqv, qw, kw, cos, sin, pos, Hq, Hkv, D, eps, qk_norm)


# ---------------------------------------------------------------- embedding
class EmbeddingFn(torch.autograd.Function):
    """Token embedding lookup.  Backward sorts the ids and sums runs of equal
    ids per warp before one vector atomic per run.

    Tied LM head: the forward marks ``table``; the fused cross-entropy that
    later uses the same tensor as its output weight then keeps its fp32
    weight gradient for this backward (``table._cfb_pending_grad``), which adds
    the embedding gradient into it and returns the sum with one cast, instead
    of a zero-filled fp32 table, two casts and autograd's add of two bf16
    gradients.
    """

    @staticmethod
    def forward(ctx, ids, table):
        C = require()
        ids_c = _c(ids.long())
        out = torch.empty(*ids.shape, table.shape[1], device=table.device, dtype=table.dtype)
        C.embedding_fwd(ids_c, _c(table), out)
        ctx.save_for_backward(ids_c)
        ctx.vshape = table.shape
        ctx.dtype = table.dtype
        ctx.table = table
        if ctx.needs_input_grad[1]:
            table._cfb_embedding_pending = True
        return out

    @staticmethod
    def backward(ctx, dy):
        C = require()
        (ids,) = ctx.saved_tensors
        table = ctx.table
        dtable = getattr(table, "_cfb_pending_grad", None)
        table._cfb_pending_grad = None
        table._cfb_embedding_pending = False
        if dtable is None or tuple(dtable.shape) != tuple(ctx.vshape):
            dtable = torch.zeros(ctx.vshape, device=dy.device, dtype=torch.float32)
        H = ctx.vshape[1]
        if H <= 1024:
            sorted_ids, order = torch.sort(ids.reshape(-1))
            C.embedding_bwd_sorted(sorted_ids, order, _c(dy), dtable)
        else:
            C.embedding_bwd(ids, _c(dy), dtable)
        return None, dtable.to(ctx.dtype)


def embedding(ids, table):
    return EmbeddingFn.apply(ids, table)


# -------------------------------------------------- fused linear cross-entropy
class LinearCrossEntropyFn(torch.autograd.Function):
    """Mean next-token CE of ``hidden @ weight.T`` without a persistent logits tensor.

    Rows are processed in chunks: one tcgen05 GEMM writes the bf16 logits of a
    chunk and per-(row, 128-column) max/sum-exp partials; one kernel turns
    them into the row loss and overwrites the logits with d(loss)/d(logits);
    two GEMMs then produce d(hidden) for the chunk and accumulate d(weight) in
    fp32.  Gradients are computed in forward (the loss is the last op of the
    graph) and scaled by the incoming gradient in backward.  Reference
    counterpart: Liger's fused linear cross-entropy used by
    complexity/core/losses/fused_ce.py:138-161.
    """

    @staticmethod
    def forward(ctx, hidden, weight, targets, ignore_index, chunk_rows):
        C = require()
        H = hidden.shape[-1]
        h = _c(hidden.reshape(-1, H))
        t = _c(targets.reshape(-1).long())
        w = _c(weight)
        T, V = h.shape[0], w.shape[0]
        valid = (t != ignore_index).sum().clamp_min(1).float()
        scale = (1.0 / valid).reshape(1)
        dh = torch.empty_like(h)
        dw = torch.zeros(V, H, device=h.device, dtype=torch.float32)
        losses = torch.empty(T, device=h.device, dtype=torch.float32)
        bn = 256
        nt = 2 * ((V + bn - 1) // bn)  # one partial per 128-column half tile
        chunk = max(128, min(T, int(chunk_rows)))
        logits = torch.empty(chunk, V, device=h.device, dtype=torch.bfloat16)
        stats = torch.empty(chunk, nt, 2, device=h.device, dtype=torch.float32)
        for r0 in range(0, T, chunk):
            r1 = min(T, r0 + chunk)
            n = r1 - r0
            hc = h[r0:r1]
            lg = logits[:n]
            C.gemm(hc, False, w, False, n, V, H, EPI_CE_STATS, out=lg, stats=stats, bn=bn)
            C.ce_loss_grad(lg, stats, nt, t[r0:r1], losses[r0:r1], scale, ignore_index)
            C.gemm(lg, False, w, True, n, H, V, EPI_STORE, out=dh[r0:r1])
            C.gemm(lg, True, hc, True, V, H, n, EPI_F32_ACC, out=dw)
        loss = losses.sum() * scale[0]
        ctx.save_for_backward(dh, dw)
        ctx.hshape = hidden.shape
        ctx.wdtype = weight.dtype
        # tied LM head: hand the fp32 weight gradient to the embedding backward
        # (the mark is consumed: one hand-off per embedding forward)
        ctx.tied = weight if getattr(weight, "_cfb_embedding_pending", False) else None
        if ctx.tied is not None:
            weight._cfb_embedding_pending = False
        return loss

    @staticmethod
    def backward(ctx, gout):
        dh, dw = ctx.saved_tensors
        dhidden = (dh * gout.to(dh.dtype)).view(ctx.hshape)
        if ctx.tied is not None:
            prev = getattr(ctx.tied, "_cfb_pending_grad", None)
            dw.mul_(gout.float())
            ctx.tied._cfb_pending_grad = dw if prev is None else prev.add_(dw)
            return dhidden, None, None, None, None
        dweight = (dw * gout.float()).to(ctx.wdtype)
        return dhidden, dweight, None, None, None


def linear_cross_entropy(hidden, weight, targets, ignore_index: int = -100,
                         chunk_rows: int = 65536):
    return LinearCrossEntropyFn.apply(hidden, weight, targets, ignore_index, chunk_rows)
