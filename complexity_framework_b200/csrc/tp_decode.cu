// Tensor-parallel decode all-reduce fused with the residual add, over NVLink
// peer memory (one process per GPU, up to 8 ranks in one NVSwitch domain).
//
// In a tensor-parallel decoder layer every rank ends attention and the FFN
// with a partial [N, H] (its heads' / its columns' share of o_proj and of the
// down projection); the layer output is residual + the sum of the partials.
// Decode steps have few rows (N <= a few hundred), so the collective is
// latency-bound: one kernel does it all.
//
//   * each rank's GEMM writes its partial into its own symmetric buffer of
//     the call site (one buffer per call site, so a buffer is rewritten only
//     after every peer passed the next call's barrier, i.e. finished reading);
//   * block 0 announces "partial ready" on every peer's signal pad (system
//     fence + release stores); every block then waits, bounded by
//     %globaltimer, until all ranks announced the same epoch;
//   * every rank reads the partials of all ranks (16-byte loads over NVLink,
//     summed in fp32 in rank order, so all ranks produce bit-identical
//     results), adds the residual and writes the bf16 output locally;
//   * the last block to finish (ticket) advances the device epoch counter, so
//     a CUDA graph that captured many calls replays with fresh epochs.
//
// With a multicast (NVLS) address the sum is one multimem.ld_reduce per
// 16 bytes instead of `world` unicast loads: the NVSwitch adds the ranks'
// values in flight.
// On timeout the kernel records kErrPeerTimeout (site = rank * 100 + peer) in
// the error word and returns without writing.
#include <cuda_bf16.h>

#include "common.cuh"
#include "tp_decode.h"

namespace cfb {
namespace {

__device__ __forceinline__ uint4 multimem_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile(
      "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(mc)
      : "memory");
  return r;
}

__global__ void __launch_bounds__(256)
    tp_allreduce_kernel(TpArPtrs pp, const __nv_bfloat16* __restrict__ resid,
                        __nv_bfloat16* __restrict__ out, int64_t n, int* epoch_dev, int* ticket,
                        int* err) {
  __shared__ int ok, e_s;
  if (threadIdx.x == 0) {
    const int e = __ldcg(epoch_dev) + 1;
    e_s = e;
    if (blockIdx.x == 0) sys_announce(pp.pad, pp.world, pp.rank, 0, e);
    ok = sys_wait_all(pp.pad, pp.world, pp.rank, 0, e, nullptr, err, pp.rank) ? 1 : 0;
  }
  __syncthreads();
  if (ok) {
    const int64_t nv = n / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      float s[8];
      if (pp.mc != nullptr) {
        const uint4 w = multimem_ld_reduce_bf16x8(pp.mc + i * 8);
        const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z),
                     d = unpack_bf16x2(w.w);
        s[0] = a.x; s[1] = a.y; s[2] = b.x; s[3] = b.y;
        s[4] = c.x; s[5] = c.y; s[6] = d.x; s[7] = d.y;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] = 0.f;
        for (int p = 0; p < pp.world; ++p) {
          const uint4 w = __ldcv(reinterpret_cast<const uint4*>(pp.buf[p] + i * 8));
          const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z),
                       d = unpack_bf16x2(w.w);
          s[0] += a.x; s[1] += a.y; s[2] += b.x; s[3] += b.y;
          s[4] += c.x; s[5] += c.y; s[6] += d.x; s[7] += d.y;
        }
      }
      if (resid != nullptr) {
        const uint4 r = *reinterpret_cast<const uint4*>(resid + i * 8);
        const float2 a = unpack_bf16x2(r.x), b = unpack_bf16x2(r.y), c = unpack_bf16x2(r.z),
                     d = unpack_bf16x2(r.w);
        s[0] += a.x; s[1] += a.y; s[2] += b.x; s[3] += b.y;
        s[4] += c.x; s[5] += c.y; s[6] += d.x; s[7] += d.y;
      }
      uint4 o;
      o.x = pack_bf16x2(s[0], s[1]);
      o.y = pack_bf16x2(s[2], s[3]);
      o.z = pack_bf16x2(s[4], s[5]);
      o.w = pack_bf16x2(s[6], s[7]);
      *reinterpret_cast<uint4*>(out + i * 8) = o;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1) {
      *ticket = 0;
      __threadfence();
      atomicExch(epoch_dev, e_s);
    }
  }
}

}  // namespace

int tp_allreduce(const TpArPtrs& pp, const __nv_bfloat16* resid, __nv_bfloat16* out, int64_t n,
                 int* epoch_dev, int* ticket, int num_sms, cudaStream_t s, int* err) {
  if (pp.world < 1 || pp.world > kTpMaxRanks || pp.rank < 0 || pp.rank >= pp.world) return -2;
  if (n % 8) return -3;
  for (int p = 0; p < pp.world; ++p)
    if (reinterpret_cast<uintptr_t>(pp.buf[p]) % 16) return -4;
  if (reinterpret_cast<uintptr_t>(out) % 16 || reinterpret_cast<uintptr_t>(resid) % 16) return -4;
  const int64_t nv = n / 8;
  int64_t grid = (nv + 255) / 256;
  if (grid > num_sms) grid = num_sms;  // co-resident: block 0 always runs with the others
  if (grid < 1) grid = 1;
  tp_allreduce_kernel<<<static_cast<int>(grid), 256, 0, s>>>(pp, resid, out, n, epoch_dev, ticket,
                                                             err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
