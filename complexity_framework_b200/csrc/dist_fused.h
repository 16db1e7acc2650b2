// Host interface of the fused data-parallel reduce + AdamW kernels (dist_fused.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cfb {

constexpr int kMaxRanks = 8;

// Pointers into every rank's symmetric buffers (index = rank in the group).
struct PeerPtrs {
  const __nv_bfloat16* grad[kMaxRanks];  // flat bf16 gradients
  __nv_bfloat16* param[kMaxRanks];       // flat bf16 parameters
  int* pad[kMaxRanks];                   // signal pads: 3 rounds x kMaxRanks ints
  float* slots[kMaxRanks];               // per-rank partial squared norms (kMaxRanks floats)
  int world;
  int rank;
};

// epoch_dev (optional): device step counter; the launch's epoch is then
// *epoch_dev * 16 + epoch.  hyper (optional): device (lr, bc1, bc2).
int fused_epoch_bump(int* epoch_dev, cudaStream_t s);
int fused_reduce_shard(const PeerPtrs& pp, int64_t lo, int64_t n, __nv_bfloat16* gs,
                       float* sumsq_local,
                       int* ticket, int epoch, const int* epoch_dev, bool publish, int num_sms,
                       cudaStream_t s, int* err);
int fused_adamw_shard(const PeerPtrs& pp, int64_t lo, int64_t n, float* master, float* m, float* v,
                      const __nv_bfloat16* gs, float lr, float b1, float b2, float eps, float wd,
                      float bc1,
                      float bc2, float max_norm, float* norm_out, int* ticket, int epoch,
                      const int* epoch_dev, const float* hyper, int num_sms, cudaStream_t s,
                      int* err);

}  // namespace cfb
