// Host interface of the sm_100a flash-attention kernels.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "gemm_tc.h"

namespace cfb {

// A [B, H, S, D] bf16 tensor given by its base pointer and element strides of
// b, h and s (d is contiguous).  Head-major storage: sb = H*S*D, sh = S*D,
// ss = D; token-major storage ([B, S, H, D] memory): sb = S*H*D, sh = D, ss = H*D.
struct Bhsd {
  void* p = nullptr;
  int64_t sb = 0, sh = 0, ss = 0;
};

// 4-D TMA map (d, s, h, b) of a Bhsd tensor: boxes of 64 x `rows` elements,
// 128-byte swizzle; rows past S read as zero.
int make_bhsd_map(CUtensorMap* m, const Bhsd& t, int B, int H, int S, int D, int rows);

// q [B,Hq,S,D], k/v [B,Hkv,S,D] (any Bhsd strides) -> out [B,S,Hq*D] bf16
// (token-major), lse [B,Hq,S] fp32 (natural log).
int flash_fwd_launch(const Bhsd& q, const Bhsd& k, const Bhsd& v, void* out, float* lse, int B,
                     int Hq, int Hkv, int S, int D, float scale, bool causal, cudaStream_t stream,
                     int* err);

// Backward: dq/dk/dv (any Bhsd strides; dk and dv share theirs) from q, k, v,
// the forward output o, its lse [B,Hq,S] and dout.  `workspace` holds
// flash_bwd_workspace_floats() fp32 values (Delta, log2 LSE, dQ accumulator).
int flash_bwd_pad(int S);
int64_t flash_bwd_workspace_floats(int B, int Hq, int S, int D);
int flash_bwd_launch(const Bhsd& q, const Bhsd& k, const Bhsd& v, const Bhsd& o,
                     const Bhsd& dout, const float* lse, const Bhsd& dq, const Bhsd& dk,
                     const Bhsd& dv, int B, int Hq, int Hkv, int S, int D, float scale,
                     bool causal, float* workspace, cudaStream_t stream, int* err);

}  // namespace cfb
