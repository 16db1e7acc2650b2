// Host interface of the tensor-parallel finish / barrier kernels (tp_fused.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cfb {

struct TpSync {
  int* pad[8];  // every rank's signal pad (int[rounds][8])
  int world;
  int rank;
  int round;
  int epoch;
};

// every rank's bf16 partial product [world*rows, ld] (peer pointers)
struct TpPartials {
  const __nv_bfloat16* part[8];
};

int tp_rs_finish(const TpPartials& pp, int64_t rows, int n, int64_t ld,
                 const __nv_bfloat16* residual, int64_t ldr, __nv_bfloat16* out, int64_t ldo,
                 const TpSync& sy, int num_sms, cudaStream_t s, int* err);
int tp_barrier(const TpSync& sy, cudaStream_t s, int* err);

}  // namespace cfb
