// Expert-contiguous execution of the TR-Hash routed experts (wide experts).
//
// Planner (three launches, no host synchronisation, deterministic): the k*T
// assignments a = j*T + t (route slot j of token t) are ordered by expert,
// stably (assignment order within an expert), into segments that start on
// 256-row boundaries, the row tile of the grouped GEMMs:
//   moe_count_k   per 1024-assignment block: histogram over experts
//   moe_scan_k    expert counts, padded segment starts, per-block write offsets,
//                 the expert of every 256-row tile (-1 past the end), padding rows
//   moe_scatter_k each assignment's row: block offset + rank among the earlier
//                 assignments of the same expert in its block (warp match + popc)
// Outputs: row_token[row] (token of a sorted row, -1 for padding), row_weight[row]
// (route weight of its slot, 0 for padding), token_pos[a] (row of assignment a),
// seg_start[E+1], tile_group[rows / 256].
//
// Gather / combine move rows between token order and expert order:
//   moe_gather_k   dst[row] = scale * src[row_token[row]]   (zero rows for padding)
//   moe_combine_k  out[t] = base[t] + scale * sum_j src[token_pos[j*T + t]]
//
// Reference counterparts: sort_pair_hash_by_expert and the scatter/reduce
// kernels K9-K12 in complexity_cuda/triton_token_routed.py:2205-2351,279-330.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace cfb {
namespace {

constexpr int kPlanBlock = 1024;
constexpr int kSegPad = 256;

__global__ void moe_count_k(const int64_t* __restrict__ routes, int64_t n, int E,
                            int* __restrict__ blk_hist) {
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t a = static_cast<int64_t>(blockIdx.x) * kPlanBlock + threadIdx.x;
  if (a < n) {
    const int64_t e = routes[a];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) blk_hist[blockIdx.x * E + e] = hist[e];
}

// one block: counts, padded segment starts, exclusive per-block offsets (in
// place over blk_hist), tile groups and padding rows
__global__ void moe_scan_k(int* __restrict__ blk_hist, int nblk, int E, int rows_bound,
                           int* __restrict__ seg_start, int* __restrict__ tile_group,
                           int* __restrict__ row_token, float* __restrict__ row_weight) {
  extern __shared__ int sh[];
  int* counts = sh;          // [E]
  int* start = sh + E;       // [E + 1]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int b = 0; b < nblk; ++b) c += blk_hist[b * E + e];
    counts[e] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int e = 0; e < E; ++e) {
      start[e] = s;
      s += (counts[e] + kSegPad - 1) / kSegPad * kSegPad;
    }
    start[E] = s;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) seg_start[e] = start[e];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int off = start[e];
    for (int b = 0; b < nblk; ++b) {
      const int c = blk_hist[b * E + e];
      blk_hist[b * E + e] = off;
      off += c;
    }
  }
  const int total = start[E];
  for (int i = threadIdx.x; i < rows_bound / kSegPad; i += blockDim.x) {
    const int r0 = i * kSegPad;
    int g = -1;
    if (r0 < total)
      for (int e = 0; e < E; ++e)
        if (r0 >= start[e] && r0 < start[e + 1]) g = e;
    tile_group[i] = g;
  }
  // padding rows inside segments and every row past the last segment
  for (int r = threadIdx.x; r < rows_bound; r += blockDim.x) {
    bool pad = r >= total;
    if (!pad)
      for (int e = 0; e < E; ++e)
        if (r >= start[e] + counts[e] && r < start[e + 1]) pad = true;
    if (pad) {
      row_token[r] = -1;
      row_weight[r] = 0.f;
    }
  }
}

__global__ void moe_scatter_k(const int64_t* __restrict__ routes, int64_t n, int64_t T, int E,
                              const int* __restrict__ blk_off, const float* __restrict__ slot_w,
                              int* __restrict__ row_token, float* __restrict__ row_weight,
                              int* __restrict__ token_pos) {
  extern __shared__ int sw[];  // [32 warps][E] counts, then exclusive offsets
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) sw[i] = 0;
  __syncthreads();
  const int64_t a = static_cast<int64_t>(blockIdx.x) * kPlanBlock + threadIdx.x;
  int e = -1;
  if (a < n) {
    const int64_t r = routes[a];
    e = (r >= 0 && r < E) ? static_cast<int>(r) : -1;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) sw[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int off = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = sw[w * E + x];
      sw[w * E + x] = off;
      off += c;
    }
  }
  __syncthreads();
  if (e >= 0) {
    const int pos = blk_off[blockIdx.x * E + e] + sw[warp * E + e] + rank;
    const int64_t t = a % T;
    row_token[pos] = static_cast<int>(t);
    row_weight[pos] = slot_w[a / T];
    token_pos[a] = pos;
  } else if (a < n) {
    token_pos[a] = -1;  // an assignment outside [0, E) has no row
  }
}

// 8 bf16 per thread, grid-stride over rows x (H / 8)
__global__ void moe_gather_k(const __nv_bfloat16* __restrict__ src, const int* __restrict__ row_token,
                             __nv_bfloat16* __restrict__ dst, int64_t rows, int H, float scale) {
  const int vec = H / 8;
  const int64_t n = rows * vec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec;
    const int c = static_cast<int>(i % vec);
    const int t = row_token[r];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t >= 0) {
      v = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(t) * H)[c];
      if (scale != 1.f) {
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(w[q]);
          w[q] = pack_bf16x2(f.x * scale, f.y * scale);
        }
      }
    }
    reinterpret_cast<uint4*>(dst + r * H)[c] = v;
  }
}

__global__ void moe_combine_k(const __nv_bfloat16* __restrict__ src, const int* __restrict__ token_pos,
                              const __nv_bfloat16* __restrict__ base, __nv_bfloat16* __restrict__ out,
                              int64_t T, int H, int k, float scale) {
  const int vec = H / 8;
  const int64_t n = T * vec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec;
    const int c = static_cast<int>(i % vec);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int pos = token_pos[j * T + t];
      if (pos < 0) continue;  // an assignment without a row contributes nothing
      const uint4 v = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(pos) * H)[c];
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(w[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    float b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (base != nullptr) {
      const uint4 v = reinterpret_cast<const uint4*>(base + t * H)[c];
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(w[q]);
        b[2 * q] = f.x;
        b[2 * q + 1] = f.y;
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      ow[q] = pack_bf16x2(b[2 * q] + scale * acc[2 * q], b[2 * q + 1] + scale * acc[2 * q + 1]);
    reinterpret_cast<uint4*>(out + t * H)[c] = o;
  }
}

int grid_for(int64_t work, int num_sms) {
  const int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace

int moe_rows_bound(int64_t n_assign, int E) {
  return static_cast<int>((n_assign + static_cast<int64_t>(E) * (kSegPad - 1) + kSegPad - 1) /
                          kSegPad * kSegPad);
}

int moe_plan_launch(const int64_t* routes, int k, int64_t T, int E, const float* slot_w,
                    int* blk_hist, int* seg_start, int* tile_group, int* row_token,
                    float* row_weight, int* token_pos, cudaStream_t stream) {
  if (E <= 0 || E > 256 || k <= 0 || T <= 0) return -2;
  const int64_t n = k * T;
  const int nblk = static_cast<int>((n + kPlanBlock - 1) / kPlanBlock);
  const int rows = moe_rows_bound(n, E);
  moe_count_k<<<nblk, kPlanBlock, E * sizeof(int), stream>>>(routes, n, E, blk_hist);
  moe_scan_k<<<1, 1024, (2 * E + 1) * sizeof(int), stream>>>(blk_hist, nblk, E, rows, seg_start,
                                                              tile_group, row_token, row_weight);
  moe_scatter_k<<<nblk, kPlanBlock, 32 * E * sizeof(int), stream>>>(
      routes, n, T, E, blk_hist, slot_w, row_token, row_weight, token_pos);
  return static_cast<int>(cudaGetLastError());
}

int moe_gather_launch(const void* src, const int* row_token, void* dst, int64_t rows, int H,
                      float scale, int num_sms, cudaStream_t stream) {
  if (H % 8) return -2;
  moe_gather_k<<<grid_for(rows * (H / 8), num_sms), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(src), row_token, static_cast<__nv_bfloat16*>(dst), rows,
      H, scale);
  return static_cast<int>(cudaGetLastError());
}

int moe_combine_launch(const void* src, const int* token_pos, const void* base, void* out,
                       int64_t T, int H, int k, float scale, int num_sms, cudaStream_t stream) {
  if (H % 8) return -2;
  moe_combine_k<<<grid_for(T * (H / 8), num_sms), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(src), token_pos,
      static_cast<const __nv_bfloat16*>(base), static_cast<__nv_bfloat16*>(out), T, H, k, scale);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
