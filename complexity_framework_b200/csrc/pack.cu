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

constexpr int kVecPerThread = 8;                    // 8-element vectors per thread per unit
constexpr int kVecUnit = 256 * kVecPerThread;        // vectors per work unit

// Row copies with unit column stride on both sides: one work unit is
// kVecUnit 8-element vectors, all loads issued before the stores (values held
// as packed bf16).
__device__ void copy_vec_unit(const CopyJob& J, int64_t unit) {
  const int vpr = J.cols / 8;  // vectors per row
  const int64_t items = (int64_t)J.rows * vpr;
  uint4 q[kVecPerThread];
  int64_t dst_o[kVecPerThread];
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k) {
    const int64_t it = unit * kVecUnit + k * 256 + threadIdx.x;
    dst_o[k] = -1;
    if (it < items) {
      const int r = static_cast<int>(it / vpr);
      const int c = static_cast<int>(it - (int64_t)r * vpr) * 8;
      const int64_t so = row_off(r, J.s_div, J.s_hi, J.s_lo) + c;
      dst_o[k] = row_off(r, J.d_div, J.d_hi, J.d_lo) + c;
      if (J.src_f32) {
        const float* f = static_cast<const float*>(J.src) + so;
        const float4 a = *reinterpret_cast<const float4*>(f);
        const float4 b = *reinterpret_cast<const float4*>(f + 4);
        q[k].x = pack_bf16x2(a.x, a.y);
        q[k].y = pack_bf16x2(a.z, a.w);
        q[k].z = pack_bf16x2(b.x, b.y);
        q[k].w = pack_bf16x2(b.z, b.w);
      } else {
        q[k] = *reinterpret_cast<const uint4*>(static_cast<const bf16*>(J.src) + so);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kVecPerThread; ++k)
    if (dst_o[k] >= 0) *reinterpret_cast<uint4*>(J.dst + dst_o[k]) = q[k];
}

// Strided (transposing) copies: one work unit is one 64 x 64 tile through
// shared memory, both sides accessed along their smaller stride.
__device__ void copy_tile_unit(const CopyJob& J, int64_t unit, float (*tile)[kTile + 1]) {
  const int tiles_c = (J.cols + kTile - 1) / kTile;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4 threads
  constexpr int kPer = kTile / 4;
  const bool src_cols = J.s_cs <= J.s_lo;
  const bool dst_cols = J.d_cs <= J.d_lo;
  const int r0 = static_cast<int>(unit / tiles_c) * kTile;
  const int c0 = static_cast<int>(unit % tiles_c) * kTile;
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

// All jobs' work units form one flat range [0, total); block b takes units
// b, b + gridDim.x, ...  Job i owns units [unit0[i], unit0[i + 1]).
__global__ void __launch_bounds__(256, 4) copy_jobs_k(CopyJobs jobs, int64_t total) {
  __shared__ float tile[kTile][kTile + 1];
  for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
    int j = 0;
    while (j + 1 < jobs.n && u >= jobs.j[j + 1].unit0) ++j;
    const CopyJob& J = jobs.j[j];
    if (J.vec) copy_vec_unit(J, u - J.unit0);
    else copy_tile_unit(J, u - J.unit0, tile);  // uniform per block: barriers are safe
  }
}

}  // namespace

void copy_jobs(const CopyJobs& jobs_in, cudaStream_t s) {
  CopyJobs jobs = jobs_in;
  int64_t total = 0;
  for (int i = 0; i < jobs.n; ++i) {
    CopyJob& J = jobs.j[i];
    // vector path: unit column strides, 8-element aligned rows and bases
    const uintptr_t sa = reinterpret_cast<uintptr_t>(J.src);
    const uintptr_t da = reinterpret_cast<uintptr_t>(J.dst);
    J.vec = J.s_cs == 1 && J.d_cs == 1 && J.cols % 8 == 0 && J.s_hi % 8 == 0 && J.s_lo % 8 == 0 &&
            J.d_hi % 8 == 0 && J.d_lo % 8 == 0 && sa % 16 == 0 && da % 16 == 0;
    J.unit0 = total;
    total += J.vec ? ((int64_t)J.rows * (J.cols / 8) + kVecUnit - 1) / kVecUnit
                   : (int64_t)((J.rows + kTile - 1) / kTile) * ((J.cols + kTile - 1) / kTile);
  }
  const int grid = static_cast<int>(total < 148 * 4 ? total : 148 * 4);
  copy_jobs_k<<<grid, 256, 0, s>>>(jobs, total);
}

}  // namespace cfb
