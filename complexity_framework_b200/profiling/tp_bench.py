"""Fused tensor-parallel GEMMs vs NCCL collectives + GEMM (one process per GPU).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        -m complexity_framework_b200.profiling.tp_bench

Times (CUDA events, max over ranks) of
  * AG->GEMM : Y[T, N/P] = AllGather(X[T/P, H]) @ W^T
       fused  : ``ag_linear`` forward (gather inside the GEMM's TMA loads)
       nccl   : ``all_gather_into_tensor`` + the same tcgen05 GEMM
  * GEMM->RS : Out[T/P, H] = ReduceScatter(X[T, F/P] @ W^T)
       fused  : ``rs_linear`` forward (peer stores + finish kernel)
       nccl   : the tcgen05 GEMM + ``reduce_scatter_tensor``
for the TR-Hash 200M shapes at 16 x 2048 tokens.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist


def _time(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    from ..ops.fused import gemm_nt
    from ..parallel.tp_fused import TPWorkspace, ag_linear, rs_linear

    T, H, F = 32768, 896, 6656
    rows = T // world
    x_shard = torch.randn(rows, H, device="cuda").bfloat16()
    w1 = (torch.randn(F // world, H, device="cuda") / 30).bfloat16()
    h = torch.randn(T, F // world, device="cuda").bfloat16()
    w2 = (torch.randn(H, F // world, device="cuda") / 60).bfloat16()
    ws = TPWorkspace()
    full = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    out_rs = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)

    def ag_fused():
        with torch.no_grad():
            ag_linear(x_shard, w1, ws, "bench.ag")

    def ag_nccl():
        dist.all_gather_into_tensor(full, x_shard)
        gemm_nt(full, w1)

    def rs_fused():
        with torch.no_grad():
            rs_linear(h, w2, None, ws, "bench.rs")

    def rs_nccl():
        y = gemm_nt(h, w2)
        dist.reduce_scatter_tensor(out_rs, y)

    res = {"world": world, "T": T, "H": H, "F": F}
    flops_ag = 2.0 * T * H * (F // world)
    flops_rs = 2.0 * T * H * (F // world)
    for name, fn, fl in (("ag_gemm_fused", ag_fused, flops_ag), ("ag_gemm_nccl", ag_nccl, flops_ag),
                         ("gemm_rs_fused", rs_fused, flops_rs), ("gemm_rs_nccl", rs_nccl, flops_rs)):
        ms = _time(fn)
        res[name] = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1)}
    # bytes that must cross NVLink per rank: (P-1)/P of the gathered / scattered tensor
    res["ag_bytes_in_per_rank"] = (world - 1) * rows * H * 2
    res["rs_bytes_out_per_rank_fp32"] = (world - 1) * rows * H * 4
    from ..ops import check_errors

    torch.cuda.synchronize()
    check_errors(torch.cuda.current_device())  # raises if any bounded wait expired
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
