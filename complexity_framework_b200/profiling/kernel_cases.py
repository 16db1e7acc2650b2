"""Small, self-contained launches of the framework's kernels for profiling.

    python -m complexity_framework_b200.profiling.kernel_cases gemm
    python -m complexity_framework_b200.profiling.kernel_cases flash
    python -m complexity_framework_b200.profiling.kernel_cases norms

Each case runs the 200M-shape kernels (inputs larger than L2, a few GB at
most) ``--iters`` times and prints CUDA-event timings with the fraction of
the measured peaks, so the same command serves both as the plain run and
as the target of an ``ncu`` capture (``-k regex:<kernel> -c 1..3``).
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops import check_errors, require
from .timing import cuda_graph_time, cuda_time, load_measured_peaks


def _report(name, ms, flops=0.0, nbytes=0.0):
    pk = load_measured_peaks()
    rec = {"case": name, "ms": round(ms, 4)}
    if flops:
        rec["tflops"] = round(flops / ms / 1e9, 1)
        rec["tensor_frac_of_measured"] = round(flops / ms / 1e9 / pk["bf16_tflops"], 3)
    if nbytes:
        rec["gbs"] = round(nbytes / ms / 1e6, 1)
        rec["hbm_frac_of_measured"] = round(nbytes / ms / 1e6 / pk["hbm_gbs"], 3)
    print(json.dumps(rec), flush=True)


def case_gemm(iters: int) -> None:
    C = require()
    T, H, A = 16384, 896, 3328
    dev = "cuda"
    x = torch.randn(T, H, device=dev).bfloat16()
    w = (torch.randn(2 * A, H, device=dev) * 0.05).bfloat16()
    gu = torch.empty(T, 2 * A, device=dev, dtype=torch.bfloat16)
    act = torch.empty(T, A, device=dev, dtype=torch.bfloat16)
    rs = torch.rand(T, 4, device=dev)
    out = torch.empty(T, 2 * A, device=dev, dtype=torch.bfloat16)
    dW = torch.zeros(A, H, device=dev)
    fl = 2.0 * T * 2 * A * H
    _report("gemm_fwd_store", cuda_time(lambda: C.gemm(x, False, w, False, T, 2 * A, H, 0, out=out),
                                        iters), fl)
    _report("gemm_swiglu_fwd", cuda_time(lambda: C.gemm(
        x, False, w, False, T, 2 * A, H, 2, gu=gu, act=act, row_scale=rs, shared_width=3072,
        expert_width=64, n_experts=4, shared_scale=1.0), iters), fl)
    _report("gemm_wgrad_splitk", cuda_time(lambda: C.gemm(act, True, x, True, A, H, T, 7, out=dW),
                                           iters), 2.0 * T * A * H)
    # data gradient of the down projection with the SwiGLU-backward epilogue
    wd = (torch.randn(H, A, device=dev) * 0.05).bfloat16()
    dy = torch.randn(T, H, device=dev).bfloat16()
    dgu = torch.empty(T, 2 * A, device=dev, dtype=torch.bfloat16)
    _report("gemm_swiglu_bwd", cuda_time(lambda: C.gemm(
        dy, False, wd, True, T, A, H, 3, out=dgu, gu=gu, row_scale=rs, shared_width=3072,
        expert_width=64, n_experts=4, shared_scale=1.0), iters), 2.0 * T * A * H)
    # down projection with the residual-add epilogue
    res = torch.randn(T, H, device=dev).bfloat16()
    o = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
    _report("gemm_down_resid", cuda_time(lambda: C.gemm(act, False, wd, False, T, H, A, 1, out=o,
                                                         residual=res), iters), 2.0 * T * A * H)
    torch.cuda.synchronize()
    check_errors(0)


def case_gemm_bn(iters: int) -> None:
    """128- vs 256-column tiles on the TR-Hash 200M step's narrow GEMMs (N = 896 or 1152)."""
    C = require()
    T, H, A, KQV = 32768, 896, 3328, 1152
    dev = "cuda"
    r = lambda *s: (torch.randn(*s, device=dev) * 0.05).bfloat16()  # noqa: E731
    x, xk, act, dgu = r(T, H), r(T, KQV), r(T, A), r(T, 2 * A)
    wk, wd, wgu = r(KQV, H), r(H, A), r(2 * A, H)
    cases = [  # name, A, a_mn, B, b_mn, M, N, K, epi, out shape, out dtype
        ("fwd_kqv", x, False, wk, False, T, KQV, H, 0, (T, KQV), torch.bfloat16),
        ("fwd_down", act, False, wd, False, T, H, A, 0, (T, H), torch.bfloat16),
        ("dgrad_kqv", xk, False, wk, True, T, H, KQV, 0, (T, H), torch.bfloat16),
        ("dgrad_gu", dgu, False, wgu, True, T, H, 2 * A, 0, (T, H), torch.bfloat16),
        ("wgrad_gu", dgu, True, x, True, 2 * A, H, T, 7, (2 * A, H), torch.float32),
        ("wgrad_down", x, True, act, True, H, A, T, 7, (H, A), torch.float32),
        ("wgrad_kqv", xk, True, x, True, KQV, H, T, 7, (KQV, H), torch.float32),
    ]
    for name, a, amn, b, bmn, M, N, K, epi, oshape, odt in cases:
        out = torch.zeros(oshape, device=dev, dtype=odt)
        for bn in (128, 256):
            _report(f"{name}_bn{bn}", cuda_time(
                lambda: C.gemm(a, amn, b, bmn, M, N, K, epi, out=out, bn=bn), iters),
                2.0 * M * N * K)
    torch.cuda.synchronize()
    check_errors(0)


def case_flash(iters: int) -> None:
    from ..ops.flash import flash_forward

    B, Hq, Hkv, S, D = 16, 14, 2, 2048, 64
    q = torch.randn(B, Hq, S, D, device="cuda").bfloat16()
    k = torch.randn(B, Hkv, S, D, device="cuda").bfloat16()
    v = torch.randn(B, Hkv, S, D, device="cuda").bfloat16()
    fl = 4.0 * B * Hq * S * S * D / 2
    _report("flash_fwd_causal", cuda_time(lambda: flash_forward(q, k, v, True, D ** -0.5), iters), fl)
    torch.cuda.synchronize()
    check_errors(0)


def case_norms(iters: int) -> None:
    C = require()
    T, H = 32768, 896
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda").bfloat16()
    y = torch.empty_like(x)
    rstd = torch.empty(T, device="cuda")
    nbytes = 2.0 * T * H * 2
    _report("rmsnorm_fwd", cuda_time(lambda: C.rmsnorm_fwd(x, w, y, rstd, 1e-6), iters),
            nbytes=nbytes)
    dy = torch.randn_like(x)
    dx = torch.empty_like(x)
    dw = torch.empty(H, device="cuda", dtype=torch.bfloat16)  # written by the last block
    _report("rmsnorm_bwd_resid", cuda_time(
        lambda: C.rmsnorm_bwd(dy, x, w, rstd, dy, dx, dw), iters), nbytes=4.0 * T * H * 2)
    B, S, Hq, Hkv, D = 16, 2048, 14, 2, 64
    kqv = torch.randn(B, S, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    qw = torch.ones(D, device="cuda").bfloat16()
    fr = torch.outer(torch.arange(S, device="cuda").float(),
                     1.0 / (10000 ** (torch.arange(0, D, 2, device="cuda").float() / D)))
    cos, sin = fr.cos().contiguous(), fr.sin().contiguous()
    pos = torch.arange(S, device="cuda", dtype=torch.int32).repeat(B, 1).contiguous()
    q = torch.empty(B, S, Hq, D, device="cuda", dtype=torch.bfloat16)  # token-major
    k = torch.empty(B, Hkv, S, D, device="cuda", dtype=torch.bfloat16)
    v = torch.empty_like(k)
    rs = torch.empty(B * S, Hq + Hkv, device="cuda")
    nb = 2.0 * kqv.numel() * 2
    _report("qk_norm_rope_fwd", cuda_time(lambda: C.qk_norm_rope_fwd(
        kqv, qw, qw, cos, sin, pos, q, k, v, rs, B, S, Hq, Hkv, D, 1e-6, True, True), iters), nbytes=nb)
    dk = torch.empty_like(kqv)
    dqw = torch.empty(D, device="cuda", dtype=torch.bfloat16)
    dkw = torch.empty(D, device="cuda", dtype=torch.bfloat16)
    _report("qk_norm_rope_bwd", cuda_time(lambda: C.qk_norm_rope_bwd(
        q, k, v, kqv, qw, qw, cos, sin, pos, rs, dk, dqw, dkw, B, S, Hq, Hkv, D, True, True), iters),
        nbytes=3.0 * kqv.numel() * 2)
    torch.cuda.synchronize()
    check_errors(0)


def _zipf_ids(T, V, seed=0, s=1.1):
    g = torch.Generator().manual_seed(seed)
    p = torch.arange(1, V + 1, dtype=torch.float64).pow(-s)
    order = torch.randperm(V, generator=g)
    return order[torch.multinomial(p / p.sum(), T, replacement=True, generator=g)]


def case_moe(iters: int) -> None:
    """One TR-Hash FFN layer (shared SwiGLU + top-2 routed experts), forward + backward,
    at the expert shapes of the 1B and 7B configurations: this framework's engine
    (grouped tcgen05 kernels) and, when installed, the reference engine (its Triton
    CGGR path), same weights, Zipf(1.1) token ids."""
    import os
    import sys

    from ..tr_hash import TRHashEngine, TRHashEngineConfig

    shapes = [("1b_e16_w256", 16384, 2048, 5632, 16, 256, "token_id_balanced_hash"),
              ("7b_e8_w512", 8192, 4096, 11008, 8, 512, "modulo_cyclic")]
    ref_root = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))), "baseline", "_ref")
    ref = None
    if os.path.isdir(os.path.join(ref_root, "complexity")):
        sys.path.insert(0, ref_root)
        try:
            import complexity.tr_hash as ref
        except Exception as exc:  # pragma: no cover - depends on the install
            print(json.dumps({"reference": f"unavailable: {exc}"}))
        finally:
            sys.path.remove(ref_root)
    for name, T, H, S, E, W, strat in shapes:
        kw = dict(hidden_size=H, vocab_size=32000, num_experts=E, top_k=2, shared_width=S,
                  expert_width=W, routing_strategy=strat, precision="bf16")
        ids = _zipf_ids(T, 32000).view(1, T).cuda()
        x = (torch.randn(1, T, H, device="cuda") * 0.5).bfloat16()
        dy = torch.randn(1, T, H, device="cuda").bfloat16()
        fl = 2.0 * 3 * T * H * (2 * S + 3 * 2 * W)   # fwd + bwd (x3) of gate|up and down GEMMs
        arms = [("ours", TRHashEngine(TRHashEngineConfig(**kw)))]
        if ref is not None:
            arms.append(("reference", ref.TRHashEngine(ref.TRHashEngineConfig(**kw))))
        for arm, eng in arms:
            eng = eng.cuda().to(torch.bfloat16)
            if arm == "reference":
                eng.load_state_dict(arms[0][1].state_dict(), strict=False)
            xx = x.clone().requires_grad_()

            def run():
                out = eng(xx, ids)
                out.backward(dy)

            ms = cuda_time(run, iters)
            _report(f"moe_fwd_bwd_{name}_{arm}", ms, fl)
    torch.cuda.synchronize()
    check_errors(0)


def case_decode(iters: int) -> None:
    """One decode step's per-layer kernels of the 7B serving benchmark: split-KV
    paged attention over 64 sequences (lengths 128..2303, GQA 32/8, D 128) and
    the skinny split-K projections (M = 64)."""
    from ..inference.paged import PagedBatch, PagePool, SeqChunk
    from ..ops import fused

    C = require()
    torch.manual_seed(0)
    g = torch.Generator().manual_seed(4321)
    lens = torch.randint(128, 2304, (64,), generator=g).tolist()
    Hq, Hkv, D = 32, 8, 128
    pool = PagePool(1, Hkv, D, sum(-(-(n + 1) // 16) for n in lens), 16,
                    dtype=torch.bfloat16, device="cuda")
    for sid, n in enumerate(lens):
        pool.allocate_sequence(sid)
        pool.reserve(sid, n + 1)
        pool.lengths[sid] = n
    pool.k.normal_()
    pool.v.normal_()
    b = PagedBatch(pool, [SeqChunk(sid, n, 1) for sid, n in enumerate(lens)])
    q = torch.randn(64, Hq, D, device="cuda").bfloat16()
    out = torch.empty_like(q)
    kv_bytes = sum(n + 1 for n in lens) * Hkv * D * 2 * 2
    _report("paged_attention_decode", cuda_time(lambda: C.paged_attention(
        q, pool.k[0], pool.v[0], b.paged_table, b.paged_cu, b.paged_kv_lens, out,
        D ** -0.5, 1), iters), nbytes=kv_bytes)
    ref = out.clone()
    for pps in (8, 12, 16, 24, 32):   # fixed splits against the automatic choice
        C.paged_attention(q, pool.k[0], pool.v[0], b.paged_table, b.paged_cu, b.paged_kv_lens,
                          out, D ** -0.5, 1, pps)
        print(json.dumps({"case": f"paged_attention_decode_pps{pps}_maxdiff",
                          "value": float((out.float() - ref.float()).abs().max())}), flush=True)
        _report(f"paged_attention_decode_pps{pps}", cuda_time(lambda: C.paged_attention(
            q, pool.k[0], pool.v[0], b.paged_table, b.paged_cu, b.paged_kv_lens, out,
            D ** -0.5, 1, pps), iters), nbytes=kv_bytes)
    x = torch.randn(64, 4096, device="cuda").bfloat16()
    for name, N, K in (("skinny_qkv", 6144, 4096), ("skinny_o", 4096, 4096),
                       ("skinny_down", 4096, 15104)):
        # enough weight copies that one graph's calls stream more than L2 (126 MB)
        copies = max(2, -(-300_000_000 // (N * K * 2)))
        ws = [(torch.randn(N, K, device="cuda") * 0.02).bfloat16() for _ in range(copies)]
        xk = x if K == 4096 else torch.randn(64, K, device="cuda").bfloat16()
        turn = [0]

        def call():
            turn[0] += 1
            return fused.gemm_nt(xk, ws[turn[0] % copies])

        # graph-replayed as in serving: eager launches of these few-microsecond
        # kernels would time the host
        _report(name, cuda_graph_time(call, iters, calls_per_graph=2 * copies),
                2.0 * 64 * N * K, nbytes=N * K * 2)
        del ws


CASES = {"decode": case_decode, "gemm": case_gemm, "gemm_bn": case_gemm_bn, "flash": case_flash, "norms": case_norms,
         "moe": case_moe}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args(argv)
    CASES[a.case](a.iters)


if __name__ == "__main__":
    main()
