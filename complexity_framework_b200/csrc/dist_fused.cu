// Data-parallel gradient reduction fused with the optimizer, over NVLink peer
// memory (one process per GPU, up to 8 ranks in one NVSwitch domain).
//
// Each rank owns shard [lo, lo+n) of a flat parameter group (ZeRO-2).  The
// flat bf16 gradient buffer and the flat bf16 parameter buffer of every rank
// live in symmetric memory, so every rank can load and store any peer's
// buffers directly.
//
//   reduce kernel : device barrier on the signal pads (all peers finished
//                   backward) -> for its shard, load the bf16 gradient slice
//                   of every peer over NVLink, sum in fp32, scale by 1/P, write
//                   the bf16 result in place over this rank's own shard (no peer
//                   reads it), accumulate the squared norm; the last block of
//                   the step publishes the norm partial into every peer's slot.
//   update kernel : device barrier (all partial norms published) -> global
//                   clip coefficient -> AdamW on the fp32 master shard ->
//                   store the new bf16 parameters straight into EVERY peer's
//                   parameter buffer (the all-gather is the optimizer's store)
//                   -> closing barrier so no rank runs its next forward before
//                   all peers' stores into its buffer have landed.
// This replaces NCCL reduce-scatter + fp32 cast + AdamW + NCCL all-gather
// (four passes and two collectives) with two kernels.
//
// Barrier epochs come either from the host or from a device step counter
// (bumped by a one-thread kernel at the start of each step), so a CUDA graph
// that captured a whole multi-GPU step advances them on every replay; the
// AdamW step likewise reads (lr, bias corrections) from a device buffer.
// Every wait on a peer is bounded by %globaltimer; on expiry the kernel
// records kErrPeerTimeout (site = waiting rank) and returns, so a missing or
// dead peer surfaces as a host-visible error instead of a hung GPU.
#include <cuda_bf16.h>

#include "common.cuh"
#include "dist_fused.h"

namespace cfb {
namespace {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_f(float* p, float v) {
  asm volatile("st.release.sys.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Announce `epoch` for this rank on round `round` of every peer's pad.
__device__ void signal_peers(const PeerPtrs& pp, int round, int epoch) {
  for (int p = 0; p < pp.world; ++p)
    st_release_sys(pp.pad[p] + round * kMaxRanks + pp.rank, epoch);
}

// Bounded wait until every rank announced `epoch` on `round` of my pad.
__device__ bool wait_peers(const PeerPtrs& pp, int round, int epoch, int* err) {
  const int* mine = pp.pad[pp.rank] + round * kMaxRanks;
  const uint64_t start = globaltimer_ns();
  for (int p = 0; p < pp.world; ++p) {
    while (ld_acquire_sys(mine + p) < epoch) {
      if (globaltimer_ns() - start > kWaitBoundNs) {
        report_error(err, kErrPeerTimeout, pp.rank * 100 + p);
        return false;
      }
    }
  }
  return true;
}

// The barrier epoch of a launch: a host value, or (graph-replayable) the
// device step counter * 16 + the launch's offset within the step.
__device__ __forceinline__ int resolve_epoch(int epoch, const int* epoch_dev) {
  return epoch_dev != nullptr ? __ldcg(epoch_dev) * 16 + epoch : epoch;
}

__global__ void epoch_bump_kernel(int* e) { e[0] += 1; }

__global__ void reduce_shard_kernel(PeerPtrs pp, int64_t lo, int64_t n,
                                    __nv_bfloat16* __restrict__ gs,
                                    float* __restrict__ sumsq_local, int* __restrict__ ticket,
                                    int epoch, const int* epoch_dev, int publish, int* err) {
  __shared__ int ok;
  __shared__ float red[32];
  epoch = resolve_epoch(epoch, epoch_dev);
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) signal_peers(pp, 0, epoch);
    ok = wait_peers(pp, 0, epoch, err) ? 1 : 0;
  }
  __syncthreads();
  float acc = 0.f;
  if (ok) {
    const float inv = 1.f / static_cast<float>(pp.world);
    const int64_t nv = n / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int p = 0; p < pp.world; ++p) {
        const uint4 w = *reinterpret_cast<const uint4*>(pp.grad[p] + lo + i * 8);
        const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z),
                     d = unpack_bf16x2(w.w);
        s[0] += a.x; s[1] += a.y; s[2] += b.x; s[3] += b.y;
        s[4] += c.x; s[5] += c.y; s[6] += d.x; s[7] += d.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] *= inv;
      uint4 w;
      w.x = pack_bf16x2(s[0], s[1]);
      w.y = pack_bf16x2(s[2], s[3]);
      w.z = pack_bf16x2(s[4], s[5]);
      w.w = pack_bf16x2(s[6], s[7]);
      // the norm uses the bf16 values the optimizer will read
      const float2 r0 = unpack_bf16x2(w.x), r1 = unpack_bf16x2(w.y), r2 = unpack_bf16x2(w.z),
                   r3 = unpack_bf16x2(w.w);
      acc += r0.x * r0.x + r0.y * r0.y + r1.x * r1.x + r1.y * r1.y + r2.x * r2.x + r2.y * r2.y +
             r3.x * r3.x + r3.y * r3.y;
      // this rank's shard of its own gradient buffer is read by no peer: reduce in place
      *reinterpret_cast<uint4*>(gs + i * 8) = w;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) {
      atomicAdd(sumsq_local, v);
      __threadfence();
      if (atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1) {
        // last block: every block has counted in; reset the counter for the
        // next launch and, for the last group of the step, publish the total
        *ticket = 0;
        if (publish) {
          __threadfence();
          const float total = atomicExch(sumsq_local, 0.f);
          for (int p = 0; p < pp.world; ++p) st_release_sys_f(pp.slots[p] + pp.rank, total);
        }
      }
    }
  }
}

__global__ void adamw_shard_kernel(PeerPtrs pp, int64_t lo, int64_t n, float* __restrict__ master,
                                   float* __restrict__ m, float* __restrict__ v,
                                   const __nv_bfloat16* __restrict__ gs, float lr, float b1, float b2,
                                   float eps, float wd, float bc1, float bc2_sqrt, float max_norm,
                                   float* __restrict__ norm_out, int* __restrict__ ticket,
                                   int epoch, const int* epoch_dev, const float* hyper,
                                   int* err) {
  __shared__ int ok;
  __shared__ float coef;
  epoch = resolve_epoch(epoch, epoch_dev);
  if (hyper != nullptr) {  // (lr, bias correction 1, bias correction 2) of this step
    lr = hyper[0];
    bc1 = hyper[1];
    bc2_sqrt = sqrtf(hyper[2]);
  }
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) signal_peers(pp, 1, epoch);
    ok = wait_peers(pp, 1, epoch, err) ? 1 : 0;
    float ss = 0.f;
    for (int p = 0; p < pp.world; ++p) ss += pp.slots[pp.rank][p];
    const float nrm = sqrtf(ss);
    coef = max_norm > 0.f ? fminf(1.f, max_norm / (nrm + 1e-6f)) : 1.f;
    if (blockIdx.x == 0 && norm_out != nullptr) *norm_out = nrm;
  }
  __syncthreads();
  if (ok) {
    const float step = lr / bc1;
    const float decay = 1.f - lr * wd;
    const int64_t nv = n / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const uint4 gw = *reinterpret_cast<const uint4*>(gs + i * 8);
      const float2 g0 = unpack_bf16x2(gw.x), g1 = unpack_bf16x2(gw.y), g2 = unpack_bf16x2(gw.z),
                   g3 = unpack_bf16x2(gw.w);
      const float g[8] = {g0.x, g0.y, g1.x, g1.y, g2.x, g2.y, g3.x, g3.y};
      float4* m4 = reinterpret_cast<float4*>(m + i * 8);
      float4* v4 = reinterpret_cast<float4*>(v + i * 8);
      float4* p4 = reinterpret_cast<float4*>(master + i * 8);
      float mm[8], vv[8], pp8[8];
      *reinterpret_cast<float4*>(mm) = m4[0];
      *reinterpret_cast<float4*>(mm + 4) = m4[1];
      *reinterpret_cast<float4*>(vv) = v4[0];
      *reinterpret_cast<float4*>(vv + 4) = v4[1];
      *reinterpret_cast<float4*>(pp8) = p4[0];
      *reinterpret_cast<float4*>(pp8 + 4) = p4[1];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float gj = g[j] * coef;
        mm[j] = b1 * mm[j] + (1.f - b1) * gj;
        vv[j] = b2 * vv[j] + (1.f - b2) * gj * gj;
        pp8[j] = pp8[j] * decay - step * mm[j] / (sqrtf(vv[j]) / bc2_sqrt + eps);
      }
      m4[0] = *reinterpret_cast<float4*>(mm);
      m4[1] = *reinterpret_cast<float4*>(mm + 4);
      v4[0] = *reinterpret_cast<float4*>(vv);
      v4[1] = *reinterpret_cast<float4*>(vv + 4);
      p4[0] = *reinterpret_cast<float4*>(pp8);
      p4[1] = *reinterpret_cast<float4*>(pp8 + 4);
      uint4 w;
      w.x = pack_bf16x2(pp8[0], pp8[1]);
      w.y = pack_bf16x2(pp8[2], pp8[3]);
      w.z = pack_bf16x2(pp8[4], pp8[5]);
      w.w = pack_bf16x2(pp8[6], pp8[7]);
      for (int p = 0; p < pp.world; ++p)
        *reinterpret_cast<uint4*>(pp.param[p] + lo + i * 8) = w;
    }
  }
  // closing barrier: my stores into every peer are complete before I signal
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1) {
      __threadfence_system();
      *ticket = 0;
      signal_peers(pp, 2, epoch);
      wait_peers(pp, 2, epoch, err);
    }
  }
}

}  // namespace

int fused_epoch_bump(int* epoch_dev, cudaStream_t s) {
  epoch_bump_kernel<<<1, 1, 0, s>>>(epoch_dev);
  return static_cast<int>(cudaGetLastError());
}

int fused_reduce_shard(const PeerPtrs& pp, int64_t lo, int64_t n, __nv_bfloat16* gs,
                       float* sumsq_local,
                       int* ticket, int epoch, const int* epoch_dev, bool publish, int num_sms,
                       cudaStream_t s, int* err) {
  if (pp.world < 1 || pp.world > kMaxRanks || n % 8 != 0 || lo % 8 != 0) return -2;
  const int grid = num_sms;  // all blocks resident: block 0 always runs
  reduce_shard_kernel<<<grid, 512, 0, s>>>(pp, lo, n, gs, sumsq_local, ticket, epoch, epoch_dev,
                                           publish ? 1 : 0, err);
  return static_cast<int>(cudaGetLastError());
}

int fused_adamw_shard(const PeerPtrs& pp, int64_t lo, int64_t n, float* master, float* m, float* v,
                      const __nv_bfloat16* gs, float lr, float b1, float b2, float eps, float wd,
                      float bc1,
                      float bc2, float max_norm, float* norm_out, int* ticket, int epoch,
                      const int* epoch_dev, const float* hyper, int num_sms, cudaStream_t s,
                      int* err) {
  if (pp.world < 1 || pp.world > kMaxRanks || n % 8 != 0 || lo % 8 != 0) return -2;
  adamw_shard_kernel<<<num_sms, 512, 0, s>>>(pp, lo, n, master, m, v, gs, lr, b1, b2, eps, wd,
                                             bc1, sqrtf(bc2), max_norm, norm_out, ticket, epoch,
                                             epoch_dev, hyper, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
