// Tensor-parallel reduce-scatter completion and barrier kernels.
//
// Reduce-scatter: every rank's GEMM stores its bf16 partial product of ALL
// rows into its own symmetric buffer (TMA stores, local).  This kernel
// announces "my partial is complete" to every peer, waits (bounded) until
// every peer announced the same, then sums, for the rows this rank owns, the
// world partials -- its own from local memory, the peers' with 16-byte P2P
// loads over NVLink, each remote byte read once -- in fp32, adds the optional
// bf16 residual and writes the bf16 result.
//
// Barrier: announce + bounded wait on one pad round; separates the last reads
// of a symmetric buffer by peers from the next local write.
#include <cuda_bf16.h>

#include "common.cuh"
#include "tp_fused.h"

namespace cfb {
namespace {

__global__ void rs_finish_kernel(TpPartials pp, int64_t rows, int n, int64_t ld,
                                 const __nv_bfloat16* __restrict__ residual, int64_t ldr,
                                 __nv_bfloat16* __restrict__ out, int64_t ldo, TpSync sy,
                                 int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) sys_announce(sy.pad, sy.world, sy.rank, sy.round, sy.epoch);
    ok = sys_wait_all(sy.pad, sy.world, sy.rank, sy.round, sy.epoch, nullptr, err, 17) ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  const int nv = n / 8;
  const int64_t total = rows * nv;
  const int64_t row0 = static_cast<int64_t>(sy.rank) * rows;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nv;
    const int c = static_cast<int>(i - r * nv) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < sy.world; ++s) {
      const uint4 w = *reinterpret_cast<const uint4*>(pp.part[s] + (row0 + r) * ld + c);
      const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), cc = unpack_bf16x2(w.z),
                   d = unpack_bf16x2(w.w);
      acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
      acc[4] += cc.x; acc[5] += cc.y; acc[6] += d.x; acc[7] += d.y;
    }
    if (residual != nullptr) {
      const uint4 w = *reinterpret_cast<const uint4*>(residual + r * ldr + c);
      const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), cc = unpack_bf16x2(w.z),
                   d = unpack_bf16x2(w.w);
      acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
      acc[4] += cc.x; acc[5] += cc.y; acc[6] += d.x; acc[7] += d.y;
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + r * ldo + c) = o;
  }
}

__global__ void tp_barrier_kernel(TpSync sy, int* err) {
  if (threadIdx.x == 0) {
    sys_announce(sy.pad, sy.world, sy.rank, sy.round, sy.epoch);
    sys_wait_all(sy.pad, sy.world, sy.rank, sy.round, sy.epoch, nullptr, err, 18);
  }
}

}  // namespace

int tp_rs_finish(const TpPartials& pp, int64_t rows, int n, int64_t ld,
                 const __nv_bfloat16* residual, int64_t ldr, __nv_bfloat16* out, int64_t ldo,
                 const TpSync& sy, int num_sms, cudaStream_t s, int* err) {
  if (n % 8 != 0 || ld % 8 != 0) return -2;
  const int64_t work = rows * (n / 8);
  int64_t blocks = (work + 255) / 256;
  if (blocks > 8 * num_sms) blocks = 8 * num_sms;
  if (blocks < 1) blocks = 1;
  rs_finish_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(pp, rows, n, ld, residual, ldr, out,
                                                            ldo, sy, err);
  return static_cast<int>(cudaGetLastError());
}

int tp_barrier(const TpSync& sy, cudaStream_t s, int* err) {
  tp_barrier_kernel<<<1, 32, 0, s>>>(sy, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
