// Batched strided 2-D copies ("copy jobs") with an optional fp32 -> bf16 cast.
//
// Packing the TR-Hash MLP weights for the fused SwiGLU GEMMs (shared gate/up
// rows interleaved with expert rows in 128-row blocks, expert [E, H, W]
// stacks transposed to rows) and unpacking their gradients were a dozen small
// torch copy/cat/stack/permute/cast kernels per layer and direction.  One
// launch here runs up to kMaxCopyJobs jobs, each an R x C copy whose row index
// may split into (r / div, r % div) parts with their own strides: that covers
// the block interleave and the expert transposes.  Tiles of 64 x 64 go
// through shared memory so both the reads and the writes run along the unit
// stride of their side.
//
// Reference counterpart: none (the reference keeps shared and expert weights
// separate and runs them as separate GEMMs, complexity/tr_hash/engine.py).
#include "common.cuh"
#include "kernels.h"

namespace cfb {
namespace {

constexpr int kTile = 64;  // transpose tiles: 64 x 64, 16 elements per thread

__device__ __forceinline__ int64_t row_off(int r, int div, int64_t hi, int64_t lo) {
  return (int64_t)(r / div) * hi + (int64_t)(r % div) * lo;
}

// Row copies with unit column stride on both sides: 8 elements per item,
// 4 items per thread in flight.
__device__ void copy_rows_vec(const CopyJob& J) {
  const int vpr = J.cols / 8;  // vectors per row
  const int64_t items = (int64_t)J.rows * vpr;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < items;
       base += 4 * stride) {
    float v[4][8];
    int64_t dst_o[4];
    bool ok[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t it = base + u * stride;
      ok[u] = it < items;
      const int r = ok[u] ? static_cast<int>(it / vpr) : 0;
      const int c = ok[u] ? static_cast<int>(it % vpr) * 8 : 0;
      const int64_t so = row_off(r, J.s_div, J.s_hi, J.s_lo) + c;
      dst_o[u] = row_off(r, J.d_div, J.d_hi, J.d_lo) + c;
      if (J.src_f32) {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(J.src) + so);
        const float4 b =
            *reinterpret_cast<const float4*>(static_cast<const float*>(J.src) + so + 4);
        v[u][0] = a.x; v[u][1] = a.y; v[u][2] = a.z; v[u][3] = a.w;
        v[u][4] = b.x; v[u][5] = b.y; v[u][6] = b.z; v[u][7] = b.w;
      } else {
        const uint4 q = *reinterpret_cast<const uint4*>(static_cast<const bf16*>(J.src) + so);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16x2(w[k]);
          v[u][2 * k] = f.x;
          v[u][2 * k + 1] = f.y;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (!ok[u]) continue;
      uint4 q;
      q.x = pack_bf16x2(v[u][0], v[u][1]);
      q.y = pack_bf16x2(v[u][2], v[u][3]);
      q.z = pack_bf16x2(v[u][4], v[u][5]);
      q.w = pack_bf16x2(v[u][6], v[u][7]);
      *reinterpret_cast<uint4*>(J.dst + dst_o[u]) = q;
    }
  }
}

__global__ void __launch_bounds__(256) copy_jobs_k(CopyJobs jobs) {
  if (blockIdx.y >= (unsigned)jobs.n) return;
  const CopyJob& J = jobs.j[blockIdx.y];
  if (J.vec) {
    copy_rows_vec(J);
    return;
  }
  const int tiles_c = (J.cols + kTile - 1) / kTile;
  const int tiles = ((J.rows + kTile - 1) / kTile) * tiles_c;
  __shared__ float tile[kTile][kTile + 1];
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4 threads
  constexpr int kPer = kTile / 4;
  const bool src_cols = J.s_cs <= J.s_lo;  // lanes run along the smaller stride
  const bool dst_cols = J.d_cs <= J.d_lo;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int r0 = (t / tiles_c) * kTile, c0 = (t % tiles_c) * kTile;
    float v[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {  // all loads first
      const int a = ty + 4 * i;
      const int r = r0 + (src_cols ? a : tx), c = c0 + (src_cols ? tx : a);
      v[i] = 0.f;
      if (r < J.rows && c < J.cols) {
        const int64_t o = row_off(r, J.s_div, J.s_hi, J.s_lo) + (int64_t)c * J.s_cs;
        v[i] = J.src_f32 ? static_cast<const float*>(J.src)[o]
                         : __bfloat162float(static_cast<const bf16*>(J.src)[o]);
      }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int a = ty + 4 * i;
      if (src_cols) tile[a][tx] = v[i];
      else tile[tx][a] = v[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int a = ty + 4 * i;
      const int r = r0 + (dst_cols ? a : tx), c = c0 + (dst_cols ? tx : a);
      if (r < J.rows && c < J.cols)
        J.dst[row_off(r, J.d_div, J.d_hi, J.d_lo) + (int64_t)c * J.d_cs] =
            __float2bfloat16(tile[r - r0][c - c0]);
    }
    __syncthreads();
  }
}

}  // namespace

void copy_jobs(const CopyJobs& jobs_in, cudaStream_t s) {
  CopyJobs jobs = jobs_in;
  int64_t max_blocks = 1;
  for (int i = 0; i < jobs.n; ++i) {
    CopyJob& J = jobs.j[i];
    // vector path: unit column strides, 8-element aligned rows and bases
    const uintptr_t sa = reinterpret_cast<uintptr_t>(J.src), da = reinterpret_cast<uintptr_t>(J.dst);
    J.vec = J.s_cs == 1 && J.d_cs == 1 && J.cols % 8 == 0 && J.s_hi % 8 == 0 && J.s_lo % 8 == 0 &&
            J.d_hi % 8 == 0 && J.d_lo % 8 == 0 && sa % (J.src_f32 ? 32 : 16) == 0 && da % 16 == 0;
    const int64_t b = J.vec ? ((int64_t)J.rows * (J.cols / 8) + 1023) / 1024
                            : (int64_t)((J.rows + kTile - 1) / kTile) * ((J.cols + kTile - 1) / kTile);
    if (b > max_blocks) max_blocks = b;
  }
  const int gx = static_cast<int>(max_blocks < 148 * 8 ? max_blocks : 148 * 8);
  copy_jobs_k<<<dim3(gx, jobs.n), 256, 0, s>>>(jobs);
}

}  // namespace cfb
