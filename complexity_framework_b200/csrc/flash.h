// Host interface of the sm_100a flash-attention kernels.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "gemm_tc.h"

namespace cfb {

// q [B,Hq,S,D], k/v [B,Hkv,S,D] bf16 -> out [B,S,Hq*D] bf16, lse [B,Hq,S] fp32 (natural log).
int flash_fwd_launch(const void* q, const void* k, const void* v, void* out, float* lse, int B,
                     int Hq, int Hkv, int S, int D, float scale, bool causal, cudaStream_t stream,
                     int* err);

}  // namespace cfb
