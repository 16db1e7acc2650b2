// Host interface of the ZeRO-3 parameter gather (fsdp.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cfb {

constexpr int kFsdpMaxRanks = 8;

struct FsdpPeers {
  const __nv_bfloat16* shard[kFsdpMaxRanks];  // every rank's shard of the unit
  int* pad[kFsdpMaxRanks];                    // signal pads (int[rounds][8])
  int world;
  int rank;
};

// dst[0 : world*shard) = concat over ranks of shard[rank][0 : shard), after a
// bounded barrier on `round` at `epoch`.  shard: elements, a multiple of 8.
int fsdp_gather(const FsdpPeers& pp, __nv_bfloat16* dst, int64_t shard, int round, int epoch,
                int num_sms, cudaStream_t s, int* err);

}  // namespace cfb
