// Paged-KV attention for decoding and chunked prefill (sm_100a, CUDA cores).
//
// Queries of a ragged batch: q [N, Hq, D] (N new tokens of several sequences,
// sequence i owns rows [cu_q[i], cu_q[i+1])).  Keys/values live in a page pool
// k_pool/v_pool [num_pages, page, Hkv, D]; page_table [num_seqs, max_pages]
// maps a sequence's logical block to a physical page; kv_lens[i] is the
// sequence length after this step's tokens were written.  Query row t of
// sequence i sits at position kv_len - q_len + t and attends causally.
//
// One CTA per (query token, KV head) serves the whole GQA group of Hq/Hkv
// query heads, so every K/V byte is read once per token and group.  Its four
// warps split the pages; inside a warp, lanes (t, half) compute the dot
// products of page key t over half of D for all heads, lanes are then re-used
// as owners of D/32 output dims to accumulate P.V, with a per-warp online
// softmax; the four warps are merged through shared memory at the end.
// Decoding is bandwidth-bound: this reads K/V exactly once per (token, group).
// Reference counterpart: the per-token page gather + SDPA of
// complexity/inference/kv_cache.py:257-308 and gqa.py:129-150.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace cfb {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxG = 16;   // query heads per KV head

template <int D, int G, int PAGE>
__global__ void __launch_bounds__(128)
    paged_attn_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k_pool,
                      const bf16* __restrict__ v_pool, const int32_t* __restrict__ page_table,
                      const int32_t* __restrict__ cu_q, const int32_t* __restrict__ kv_lens,
                      bf16* __restrict__ out, int num_seqs, int max_pages, int Hq, int Hkv,
                      float scale_log2) {
  constexpr int DL = D / 32;        // output dims owned per lane
  constexpr int DH = D / 2;         // dims per half-warp in the score phase
  __shared__ float sq[G][D];
  __shared__ float s_m[kWarps][G], s_l[kWarps][G];
  __shared__ float s_acc[kWarps][G][D];

  const int tok = blockIdx.x;
  const int kvh = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // sequence of this token (binary search over cu_q)
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_q[mid] <= tok) lo = mid; else hi = mid - 1;
  }
  const int seq = lo;
  const int q_len = cu_q[seq + 1] - cu_q[seq];
  const int kv_len = kv_lens[seq];
  const int qpos = kv_len - q_len + (tok - cu_q[seq]);
  const int n_keys = qpos + 1;                      // causal
  const int n_pages = (n_keys + PAGE - 1) / PAGE;
  const int32_t* pt = page_table + static_cast<int64_t>(seq) * max_pages;

  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    sq[g][d] = __bfloat162float(q[(static_cast<int64_t>(tok) * Hq + kvh * G + g) * D + d]);
  }
  __syncthreads();

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < DL; ++j) acc[g][j] = 0.f;
  }
  const int key_in_page = lane & (PAGE - 1);
  const int half = lane / PAGE;                      // PAGE == 16: two halves of D

  for (int p = warp; p < n_pages; p += kWarps) {
    const int page = pt[p];
    const int key = p * PAGE + key_in_page;
    const bool valid = key < n_keys;
    // ---- scores of key `key_in_page` for every head (each half-warp covers D/2)
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (valid) {
      const bf16* kr = k_pool + ((static_cast<int64_t>(page) * PAGE + key_in_page) * Hkv + kvh) * D +
                       half * DH;
#pragma unroll
      for (int d = 0; d < DH; d += 8) {
        const uint4 w = *reinterpret_cast<const uint4*>(kr + d);
        const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z),
                     e = unpack_bf16x2(w.w);
        const float kv8[8] = {a.x, a.y, b.x, b.y, c.x, c.y, e.x, e.y};
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float* qg = &sq[g][half * DH + d];
#pragma unroll
          for (int u = 0; u < 8; ++u) s[g] += qg[u] * kv8[u];
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] += __shfl_xor_sync(0xffffffffu, s[g], PAGE);   // join the two halves of D
      s[g] = valid ? s[g] * scale_log2 : -INFINITY;
    }
    // ---- online softmax over the page's keys, per head
    float pexp[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = s[g];
#pragma unroll
      for (int o = PAGE / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m[g], mx);
      const float alpha = m[g] == -INFINITY ? 0.f : exp2f(m[g] - m_new);
      pexp[g] = valid ? exp2f(s[g] - m_new) : 0.f;
      float ps = pexp[g];
#pragma unroll
      for (int o = PAGE / 2; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[g] = l[g] * alpha + ps;
      m[g] = m_new;
#pragma unroll
      for (int j = 0; j < DL; ++j) acc[g][j] *= alpha;
    }
    // ---- P.V: lane owns dims [lane*DL, lane*DL+DL) for every head
    const int nk = min(PAGE, n_keys - p * PAGE);
    for (int t = 0; t < nk; ++t) {
      const bf16* vr = v_pool + ((static_cast<int64_t>(page) * PAGE + t) * Hkv + kvh) * D + lane * DL;
      float vv[DL];
#pragma unroll
      for (int j = 0; j < DL; j += 2) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vr + j));
        vv[j] = f.x;
        vv[j + 1] = f.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pt_g = __shfl_sync(0xffffffffu, pexp[g], t);
#pragma unroll
        for (int j = 0; j < DL; ++j) acc[g][j] += pt_g * vv[j];
      }
    }
  }
  // ---- merge the warps
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[warp][g] = m[g];
      s_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < DL; ++j) s_acc[warp][g][lane * DL + j] = acc[g][j];
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mm = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, s_m[w][g]);
    float ll = 0.f, o = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      if (s_m[w][g] == -INFINITY) continue;
      const float f = exp2f(s_m[w][g] - mm);
      ll += s_l[w][g] * f;
      o += s_acc[w][g][d] * f;
    }
    out[(static_cast<int64_t>(tok) * Hq + kvh * G + g) * D + d] =
        __float2bfloat16(ll > 0.f ? o / ll : 0.f);
  }
}

template <int D, int G>
void launch_g(const bf16* q, const bf16* k, const bf16* v, const int32_t* pt, const int32_t* cu,
              const int32_t* kl, bf16* out, int N, int num_seqs, int max_pages, int Hq, int Hkv,
              float sl2, cudaStream_t s) {
  paged_attn_kernel<D, G, 16><<<dim3(N, Hkv), 128, 0, s>>>(q, k, v, pt, cu, kl, out, num_seqs,
                                                          max_pages, Hq, Hkv, sl2);
}

template <int D>
int launch_d(const bf16* q, const bf16* k, const bf16* v, const int32_t* pt, const int32_t* cu,
             const int32_t* kl, bf16* out, int N, int num_seqs, int max_pages, int Hq, int Hkv,
             float sl2, cudaStream_t s) {
  switch (Hq / Hkv) {
    case 1: launch_g<D, 1>(q, k, v, pt, cu, kl, out, N, num_seqs, max_pages, Hq, Hkv, sl2, s); break;
    case 2: launch_g<D, 2>(q, k, v, pt, cu, kl, out, N, num_seqs, max_pages, Hq, Hkv, sl2, s); break;
    case 4: launch_g<D, 4>(q, k, v, pt, cu, kl, out, N, num_seqs, max_pages, Hq, Hkv, sl2, s); break;
    case 7: launch_g<D, 7>(q, k, v, pt, cu, kl, out, N, num_seqs, max_pages, Hq, Hkv, sl2, s); break;
    case 8: launch_g<D, 8>(q, k, v, pt, cu, kl, out, N, num_seqs, max_pages, Hq, Hkv, sl2, s); break;
    default: return -3;
  }
  return 0;
}

}  // namespace

int paged_attention(const bf16* q, const bf16* k_pool, const bf16* v_pool,
                    const int32_t* page_table, const int32_t* cu_q, const int32_t* kv_lens,
                    bf16* out, int N, int num_seqs, int max_pages, int Hq, int Hkv, int D,
                    int page_size, float scale, cudaStream_t s) {
  if (page_size != 16) return -4;
  const float sl2 = scale * 1.4426950408889634f;
  int rc;
  if (D == 64)
    rc = launch_d<64>(q, k_pool, v_pool, page_table, cu_q, kv_lens, out, N, num_seqs, max_pages,
                      Hq, Hkv, sl2, s);
  else if (D == 128)
    rc = launch_d<128>(q, k_pool, v_pool, page_table, cu_q, kv_lens, out, N, num_seqs, max_pages,
                       Hq, Hkv, sl2, s);
  else
    return -2;
  if (rc) return rc;
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
