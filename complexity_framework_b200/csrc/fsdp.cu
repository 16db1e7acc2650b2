// Fully sharded data parallelism (ZeRO-3): gather of one unit's bf16
// parameters from every rank's shard over NVLink peer memory.
//
// Each rank owns a contiguous shard of the unit's flat bf16 parameter buffer
// in symmetric memory.  Before a unit's forward (and again before its
// backward) the kernel below pulls all shards into this rank's local full
// buffer: block 0 announces on every peer's signal pad that this rank's shard
// is current for `epoch` (its optimizer step has been stream-ordered before the
// launch), every block waits (bounded by %globaltimer) until all ranks have
// announced, then copies 16-byte vectors: element e comes from rank
// e / shard.  The launch is issued on a side stream one unit ahead, so the
// gather overlaps the previous unit's compute.  The reduce-scatter of the
// gradients reuses reduce_shard_kernel (dist_fused.cu).
#include <cuda_bf16.h>

#include "common.cuh"
#include "fsdp.h"

namespace cfb {
namespace {

__global__ void __launch_bounds__(256)
    fsdp_gather_kernel(FsdpPeers pp, __nv_bfloat16* __restrict__ dst, int64_t shard, int round,
                       int epoch, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) sys_announce(pp.pad, pp.world, pp.rank, round, epoch);
    ok = sys_wait_all(pp.pad, pp.world, pp.rank, round, epoch, nullptr, err, 30 + pp.rank) ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  const int64_t per = shard / 8;  // vectors per shard
  const int64_t total = per * pp.world;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = i / per, j = i - p * per;
    const uint4 v = __ldcv(reinterpret_cast<const uint4*>(pp.shard[p]) + j);
    reinterpret_cast<uint4*>(dst)[i] = v;
  }
}

}  // namespace

int fsdp_gather(const FsdpPeers& pp, __nv_bfloat16* dst, int64_t shard, int round, int epoch,
                int num_sms, cudaStream_t s, int* err) {
  if (pp.world < 1 || pp.world > kFsdpMaxRanks || pp.rank < 0 || pp.rank >= pp.world) return -2;
  if (shard % 8) return -3;
  for (int p = 0; p < pp.world; ++p)
    if (reinterpret_cast<uintptr_t>(pp.shard[p]) % 16) return -4;
  if (reinterpret_cast<uintptr_t>(dst) % 16) return -4;
  const int64_t vecs = shard / 8 * pp.world;
  int64_t grid = (vecs + 255) / 256;
  if (grid > 2 * num_sms) grid = 2 * num_sms;  // resident: every block can reach the barrier
  if (grid < 1) grid = 1;
  fsdp_gather_kernel<<<static_cast<int>(grid), 256, 0, s>>>(pp, dst, shard, round, epoch, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
