// Tensor-parallel collectives that complete the fused GEMMs of gemm_tc.cu.
//
// Reduce-scatter: the GEMM epilogue of every rank stores its fp32 partial of
// the rows owned by rank p into p's slot array slots_p[src][rows][ld] over
// NVLink (plain stores, no atomics: the sum below is deterministic).  This
// kernel then announces "my stores are done" to every peer, waits (bounded)
// until every peer announced the same, and sums the world slots of its own
// rows in fp32 (+ optional bf16 residual) into the bf16 output.
//
// Barrier: announce + bounded wait on one pad round; used to separate the
// last reads of a symmetric buffer by peers from the next local write.
#include <cuda_bf16.h>

#include "common.cuh"
#include "tp_fused.h"

namespace cfb {
namespace {

__global__ void rs_finish_kernel(const float* __restrict__ slots, int world, int64_t rows, int n,
                                 int64_t ld, const __nv_bfloat16* __restrict__ residual,
                                 int64_t ldr, __nv_bfloat16* __restrict__ out, int64_t ldo,
                                 TpSync sy, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) sys_announce(sy.pad, sy.world, sy.rank, sy.round, sy.epoch);
    ok = sys_wait_all(sy.pad, sy.world, sy.rank, sy.round, sy.epoch, nullptr, err, 17) ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  const int nv = n / 4;
  const int64_t total = rows * nv;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nv;
    const int c = static_cast<int>(i - r * nv) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < world; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(slots + (s * rows + r) * ld + c);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if (residual != nullptr) {
      const uint2 rw = *reinterpret_cast<const uint2*>(residual + r * ldr + c);
      const float2 a = unpack_bf16x2(rw.x), b = unpack_bf16x2(rw.y);
      acc.x += a.x;
      acc.y += a.y;
      acc.z += b.x;
      acc.w += b.y;
    }
    uint2 o;
    o.x = pack_bf16x2(acc.x, acc.y);
    o.y = pack_bf16x2(acc.z, acc.w);
    *reinterpret_cast<uint2*>(out + r * ldo + c) = o;
  }
}

__global__ void tp_barrier_kernel(TpSync sy, int* err) {
  if (threadIdx.x == 0) {
    sys_announce(sy.pad, sy.world, sy.rank, sy.round, sy.epoch);
    sys_wait_all(sy.pad, sy.world, sy.rank, sy.round, sy.epoch, nullptr, err, 18);
  }
}

}  // namespace

int tp_rs_finish(const float* slots, int world, int64_t rows, int n, int64_t ld,
                 const __nv_bfloat16* residual, int64_t ldr, __nv_bfloat16* out, int64_t ldo,
                 const TpSync& sy, int num_sms, cudaStream_t s, int* err) {
  if (n % 4 != 0) return -2;
  const int64_t work = rows * (n / 4);
  int64_t blocks = (work + 255) / 256;
  if (blocks > 4 * num_sms) blocks = 4 * num_sms;
  if (blocks < 1) blocks = 1;
  rs_finish_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(slots, world, rows, n, ld, residual,
                                                            ldr, out, ldo, sy, err);
  return static_cast<int>(cudaGetLastError());
}

int tp_barrier(const TpSync& sy, cudaStream_t s, int* err) {
  tp_barrier_kernel<<<1, 32, 0, s>>>(sy, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
