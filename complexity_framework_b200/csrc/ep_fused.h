// Host interface of the expert-parallel gather / combine kernel (ep_fused.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cfb {

struct EpSources {
  const __nv_bfloat16* p[8];  // every rank's source rows [*, H]
};

struct EpSync {
  int* pad[8];
  int world;       // ranks in the barrier (0: no barrier)
  int world_srcs;  // valid entries of EpSources
  int rank;
  int round;
  int epoch;
};

int ep_gather_combine(const EpSources& srcs, const int* idx, const float* w, int64_t rows, int H,
                      int64_t stride, const __nv_bfloat16* residual, __nv_bfloat16* out, int k,
                      const EpSync& sy, int num_sms, cudaStream_t s, int* err);

}  // namespace cfb
