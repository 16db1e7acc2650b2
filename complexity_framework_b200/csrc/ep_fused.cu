// Expert-parallel dispatch / combine over NVLink peer memory.
//
// One primitive serves both directions:
//   out[i, :] = (residual[i, :]) + sum_j w[i, j] * src_{rank(idx[i,j])}[row(idx[i,j]), :]
// where idx encodes (rank, row) as rank * stride + row (negative: skipped).
// Dispatch (k = 1, w = 1): an expert owner pulls the token rows routed to its
// experts from the token owners' hidden buffers into an expert-contiguous
// buffer.  Combine (k = top-k, w = route weights, + residual): a token owner
// pulls each slot's expert output row from the expert owners and sums them.
// Rows move with 16-byte P2P loads, one warp per output row, every remote
// byte read once; no packing, no all-to-all.  Before reading peers the kernel
// announces this rank's arrival on a symmetric signal pad (its source buffer
// is complete: written by earlier kernels on this stream) and waits, bounded,
// for every peer.
#include <cuda_bf16.h>

#include "common.cuh"
#include "ep_fused.h"

namespace cfb {
namespace {

template <int K>
__global__ void gather_combine_kernel(EpSources srcs, const int* __restrict__ idx,
                                      const float* __restrict__ w, int64_t rows, int H,
                                      int64_t stride, const __nv_bfloat16* __restrict__ residual,
                                      __nv_bfloat16* __restrict__ out, int k, EpSync sy,
                                      int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    if (sy.world > 0) {
      if (blockIdx.x == 0) sys_announce(sy.pad, sy.world, sy.rank, sy.round, sy.epoch);
      ok = sys_wait_all(sy.pad, sy.world, sy.rank, sy.round, sy.epoch, nullptr, err, 21) ? 1 : 0;
    }
  }
  __syncthreads();
  if (!ok) return;
  const int lane = threadIdx.x & 31;
  const int nv = H / 8;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       i < rows; i += warps) {
    int src_rank[K > 0 ? K : 8];
    int64_t src_row[K > 0 ? K : 8];
    float wt[K > 0 ? K : 8];
    const int kk = K > 0 ? K : k;
    for (int j = 0; j < kk; ++j) {
      const int v = idx[i * kk + j];
      src_rank[j] = v < 0 ? -1 : static_cast<int>(v / stride);
      src_row[j] = v < 0 ? 0 : v % stride;
      wt[j] = w != nullptr ? w[i * kk + j] : 1.0f;
      if (src_rank[j] >= sy.world_srcs) src_rank[j] = -1;  // bounds guard
    }
    for (int c = lane; c < nv; c += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (residual != nullptr) {
        const uint4 r = *reinterpret_cast<const uint4*>(residual + i * H + c * 8);
        const float2 a = unpack_bf16x2(r.x), b = unpack_bf16x2(r.y), cc = unpack_bf16x2(r.z),
                     d = unpack_bf16x2(r.w);
        acc[0] = a.x; acc[1] = a.y; acc[2] = b.x; acc[3] = b.y;
        acc[4] = cc.x; acc[5] = cc.y; acc[6] = d.x; acc[7] = d.y;
      }
      for (int j = 0; j < kk; ++j) {
        if (src_rank[j] < 0) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(srcs.p[src_rank[j]] + src_row[j] * H +
                                                        c * 8);
        const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), cc = unpack_bf16x2(v.z),
                     d = unpack_bf16x2(v.w);
        const float s = wt[j];
        acc[0] += s * a.x; acc[1] += s * a.y; acc[2] += s * b.x; acc[3] += s * b.y;
        acc[4] += s * cc.x; acc[5] += s * cc.y; acc[6] += s * d.x; acc[7] += s * d.y;
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(out + i * H + c * 8) = o;
    }
  }
}

}  // namespace

int ep_gather_combine(const EpSources& srcs, const int* idx, const float* w, int64_t rows, int H,
                      int64_t stride, const __nv_bfloat16* residual, __nv_bfloat16* out, int k,
                      const EpSync& sy, int num_sms, cudaStream_t s, int* err) {
  if (H % 8 != 0 || k < 1 || k > 8) return -2;
  int64_t blocks = (rows + 7) / 8;  // 8 warps per block, one row per warp
  if (blocks > 16 * num_sms) blocks = 16 * num_sms;
  if (blocks < 1) blocks = 1;
  if (k == 1)
    gather_combine_kernel<1><<<static_cast<int>(blocks), 256, 0, s>>>(
        srcs, idx, w, rows, H, stride, residual, out, k, sy, err);
  else if (k == 2)
    gather_combine_kernel<2><<<static_cast<int>(blocks), 256, 0, s>>>(
        srcs, idx, w, rows, H, stride, residual, out, k, sy, err);
  else
    gather_combine_kernel<0><<<static_cast<int>(blocks), 256, 0, s>>>(
        srcs, idx, w, rows, H, stride, residual, out, k, sy, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
