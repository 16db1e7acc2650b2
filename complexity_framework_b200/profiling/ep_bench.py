"""Expert-parallel routed FFN: NVLink dispatch/combine kernels vs NCCL all-to-all.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        -m complexity_framework_b200.profiling.ep_bench

Times forward + backward of the routed experts of one TR-Hash layer
(E = 8 experts of width 512, top-2, H = 896, 16384 tokens per rank), CUDA
events, max over ranks, SM clocks sampled during each timed loop:
  * fused : ``parallel.ep_fused.FusedExpertParallelRouted`` (token ids gathered
            once, device plan, pull-based P2P dispatch / combine, grouped
            tcgen05 GEMMs over the local experts)
  * nccl  : ``parallel.expert_parallel.ExpertParallelRouted`` (all_to_all_single
            + index_select / index_add, matmuls per local expert)
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist


def main():
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    from ..ops import check_errors
    from ..parallel.ep_fused import FusedExpertParallelRouted
    from ..parallel.expert_parallel import ExpertParallelRouted
    from ..parallel.tp_fused import TPWorkspace
    from ..tr_hash.config import TRHashEngineConfig
    from ..tr_hash.engine import TRHashEngine

    H, E, W, k, T = 896, 8, 512, 2, 16384
    torch.manual_seed(0)
    eng = TRHashEngine(TRHashEngineConfig(hidden_size=H, vocab_size=32000, num_experts=E,
                                          top_k=k, shared_width=0, expert_width=W)).cuda()
    eng = eng.bfloat16()
    ids = torch.randint(0, 32000, (1, T), generator=torch.Generator().manual_seed(rank)).cuda()
    routes = eng._routes(ids).reshape(k, -1)
    x = (torch.randn(T, H, device="cuda") * 0.5).bfloat16().requires_grad_()
    gout = torch.randn(T, H, device="cuda").bfloat16()
    ws = TPWorkspace()
    fused = FusedExpertParallelRouted(eng, ws, "bench")
    nccl = ExpertParallelRouted(eng, None).cuda()

    def run(mod):
        if mod is fused:  # routes of every rank follow from the token ids
            y = mod(x, routes, eng._route_weights, token_ids=ids, route_fn=eng._routes)
        else:
            y = mod(x, routes, eng._route_weights)
        y.backward(gout)

    res = {"H": H, "E": E, "W": W, "top_k": k, "tokens_per_rank": T,
           "world": dist.get_world_size()}
    from .timing import ClockSampler

    iters = 300  # about a second per path: long enough for the clock sampler

    for name, mod in (("fused", fused), ("nccl", nccl)):
        for _ in range(3):
            run(mod)
        dist.barrier()
        torch.cuda.synchronize()
        clocks = ClockSampler(torch.cuda.current_device())
        if rank == 0:
            clocks.start()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            run(mod)
        e.record()
        torch.cuda.synchronize()
        if rank == 0:
            res[name + "_clocks"] = clocks.stop()
        ms = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        res[name + "_fwd_bwd_ms"] = round(float(ms), 4)
    check_errors(torch.cuda.current_device())
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
