// Host interface of the tensor-parallel decode all-reduce (tp_decode.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cfb {

constexpr int kTpMaxRanks = 8;

struct TpArPtrs {
  const __nv_bfloat16* buf[kTpMaxRanks];  // every rank's partial buffer of this call site
  int* pad[kTpMaxRanks];                  // signal pads (int[rounds][8]); round 0 is used
  const __nv_bfloat16* mc;                // multicast address of the buffer, or null
  int world;
  int rank;
};

// out = resid (optional) + sum over ranks of buf[rank][0:n); n a multiple of 8.
// epoch_dev / ticket: per-group device counters (int32, zero-initialised).
int tp_allreduce(const TpArPtrs& pp, const __nv_bfloat16* resid, __nv_bfloat16* out, int64_t n,
                 int* epoch_dev, int* ticket, int num_sms, cudaStream_t s, int* err);

}  // namespace cfb
