// Paged-KV attention for decoding and chunked prefill (sm_100a).
//
// Queries of a ragged batch: q [N, Hq, D] (N new tokens of several sequences,
// sequence i owns rows [cu_q[i], cu_q[i+1])).  Keys/values live in a page pool
// k_pool/v_pool [num_pages, page, Hkv, D]; page_table [num_seqs, max_pages]
// maps a sequence's logical block to a physical page; kv_lens[i] is the
// sequence length after this step's tokens were written.  Query row t of
// sequence i sits at position kv_len - q_len + t and attends causally.
//
// Decoding reads every cached K/V byte once per step, so the kernel is built
// for memory-level parallelism (split-KV "flash decoding"):
//
// * grid (split, KV head, query token): one CTA serves the whole GQA group of
//   Hq/Hkv query heads over a contiguous range of pages; a short sequence uses
//   fewer splits (CTAs past its last page exit at once), a long one spreads
//   over many SMs.  The host picks the pages per split from the batch size so
//   a decode step launches several CTAs per SM.
// * each of the four warps streams its pages (page w, w+4, ...) through a
//   two-stage cp.async ring in shared memory: the next page's 2 x 4 KB of K/V
//   is in flight while the current one is consumed.  K rows are padded by 16
//   bytes so the 16 lanes reading different keys hit different banks.
// * inside a warp, lanes (key t, half) form the dot products of page key t
//   over half of D for all heads; then lanes own D/32 output dims and
//   accumulate P.V with a per-warp online softmax (exp2 domain).
// * warps merge through shared memory; with one split the CTA writes the
//   normalised bf16 output, otherwise a normalised fp32 partial plus its
//   log2-sum-exp, and a combine kernel reduces the splits.
//
// Reference counterpart: the per-token page gather + SDPA of
// complexity/inference/kv_cache.py:257-308 and gqa.py:129-150.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace cfb {
namespace {

constexpr int kWarps = 4;
constexpr int kPage = 16;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int D>
struct PagedSmem {
  static constexpr int K_ROW = D * 2 + 16;             // bytes, padded
  static constexpr int K_BYTES = kPage * K_ROW;
  static constexpr int V_BYTES = kPage * D * 2;
  static constexpr int STAGE = K_BYTES + V_BYTES;
  static constexpr int WARP = 2 * STAGE;
  static constexpr int RING = kWarps * WARP;
};

template <int D, int G>
constexpr int paged_smem_bytes() {
  // ring (reused for the warp merge) + fp32 queries + (m, l) per warp and head
  return PagedSmem<D>::RING + G * D * 4 + 2 * kWarps * G * 4;
}

template <int D, int G>
__global__ void __launch_bounds__(128)
    paged_attn_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k_pool,
                      const bf16* __restrict__ v_pool, const int32_t* __restrict__ page_table,
                      const int32_t* __restrict__ cu_q, const int32_t* __restrict__ kv_lens,
                      bf16* __restrict__ out, float* __restrict__ ws_o,
                      float* __restrict__ ws_lse, int num_seqs, int max_pages, int Hq, int Hkv,
                      int pages_per_split, int splits, float scale_log2) {
  using S = PagedSmem<D>;
  constexpr int DL = D / 32;        // output dims owned per lane
  constexpr int DH = D / 2;         // dims per half-warp in the score phase
  constexpr int CHUNKS = D * 2 / 16;  // 16-byte chunks per K or V row
  extern __shared__ __align__(128) uint8_t smem[];
  float* sq = reinterpret_cast<float*>(smem + S::RING);          // [G][D]
  float* s_m = sq + G * D;                                        // [kWarps][G]
  float* s_l = s_m + kWarps * G;                                  // [kWarps][G]

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int tok = blockIdx.z;
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
  const int n_pages = (n_keys + kPage - 1) / kPage;
  const int p_begin = split * pages_per_split;
  const int p_end = min(n_pages, p_begin + pages_per_split);
  const int64_t orow = static_cast<int64_t>(tok) * Hq + kvh * G;
  if (p_begin >= p_end) {  // this split lies past the sequence: an empty partial
    if (splits > 1 && threadIdx.x < G) ws_lse[(orow + threadIdx.x) * splits + split] = -INFINITY;
    return;
  }
  const int32_t* pt = page_table + static_cast<int64_t>(seq) * max_pages;

  // ---- this warp's pages: p_begin + warp + kWarps * i
  const int first = p_begin + warp;
  const int count = first < p_end ? (p_end - first + kWarps - 1) / kWarps : 0;
  uint8_t* ring = smem + warp * S::WARP;
  auto issue = [&](int i) {
    const int page = __ldg(pt + first + kWarps * i);
    uint8_t* st = ring + (i & 1) * S::STAGE;
    const int64_t base = (static_cast<int64_t>(page) * kPage * Hkv + kvh) * D;
#pragma unroll
    for (int c = lane; c < kPage * CHUNKS; c += 32) {
      const int r = c / CHUNKS, x = c % CHUNKS;
      const int64_t g = base + static_cast<int64_t>(r) * Hkv * D + x * 8;
      cp_async16(st + r * S::K_ROW + x * 16, k_pool + g);
      cp_async16(st + S::K_BYTES + r * D * 2 + x * 16, v_pool + g);
    }
  };
  if (count > 0) issue(0);
  cp_async_commit();

  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    sq[i] = __bfloat162float(q[(orow + g) * D + d]);
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
  const int key_in_page = lane & (kPage - 1);
  const int half = lane / kPage;

  for (int i = 0; i < count; ++i) {
    if (i + 1 < count) issue(i + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const uint8_t* st = ring + (i & 1) * S::STAGE;
    const int p = first + kWarps * i;
    const int key = p * kPage + key_in_page;
    const bool valid = key < n_keys;
    // ---- scores of key `key_in_page` for every head (each half-warp covers D/2)
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    {
      const uint8_t* kr = st + key_in_page * S::K_ROW + half * DH * 2;
#pragma unroll
      for (int d = 0; d < DH; d += 8) {
        const uint4 w = *reinterpret_cast<const uint4*>(kr + d * 2);
        const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z),
                     e = unpack_bf16x2(w.w);
        const float kv8[8] = {a.x, a.y, b.x, b.y, c.x, c.y, e.x, e.y};
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float* qg = sq + g * D + half * DH + d;
#pragma unroll
          for (int u = 0; u < 8; ++u) s[g] = fmaf(qg[u], kv8[u], s[g]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] += __shfl_xor_sync(0xffffffffu, s[g], kPage);   // join the two halves of D
      s[g] = valid ? s[g] * scale_log2 : -INFINITY;
    }
    // ---- online softmax over the page's keys, per head
    float pexp[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = s[g];
#pragma unroll
      for (int o = kPage / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m[g], mx);
      const float alpha = m[g] == -INFINITY ? 0.f : exp2f(m[g] - m_new);
      pexp[g] = valid ? exp2f(s[g] - m_new) : 0.f;
      float ps = pexp[g];
#pragma unroll
      for (int o = kPage / 2; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l[g] = l[g] * alpha + ps;
      m[g] = m_new;
#pragma unroll
      for (int j = 0; j < DL; ++j) acc[g][j] *= alpha;
    }
    // ---- P.V: lane owns dims [lane*DL, lane*DL+DL) for every head
    const int nk = min(kPage, n_keys - p * kPage);
    const uint8_t* vs = st + S::K_BYTES + lane * DL * 2;
    for (int t = 0; t < nk; ++t) {
      float vv[DL];
#pragma unroll
      for (int j = 0; j < DL; j += 2) {
        const float2 f = __bfloat1622float2(
            *reinterpret_cast<const __nv_bfloat162*>(vs + t * D * 2 + j * 2));
        vv[j] = f.x;
        vv[j + 1] = f.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pt_g = __shfl_sync(0xffffffffu, pexp[g], t);
#pragma unroll
        for (int j = 0; j < DL; ++j) acc[g][j] = fmaf(pt_g, vv[j], acc[g][j]);
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
  }
  cp_async_wait<0>();

  // ---- merge the warps (the ring is free now)
  __syncthreads();
  float* s_acc = reinterpret_cast<float*>(smem);  // [kWarps][G][D]
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[warp * G + g] = m[g];
      s_l[warp * G + g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < DL; ++j) s_acc[(warp * G + g) * D + lane * DL + j] = acc[g][j];
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mm = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, s_m[w * G + g]);
    float ll = 0.f, o = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      if (s_m[w * G + g] == -INFINITY) continue;
      const float f = exp2f(s_m[w * G + g] - mm);
      ll += s_l[w * G + g] * f;
      o += s_acc[(w * G + g) * D + d] * f;
    }
    const float val = ll > 0.f ? o / ll : 0.f;
    if (splits == 1) {
      out[(orow + g) * D + d] = __float2bfloat16(val);
    } else {
      ws_o[((orow + g) * splits + split) * D + d] = val;
      if (d == 0) ws_lse[(orow + g) * splits + split] = ll > 0.f ? mm + log2f(ll) : -INFINITY;
    }
  }
}

// out[row, d] = sum_s o_s[d] 2^(lse_s - M) / sum_s 2^(lse_s - M); one CTA per row.
template <int D>
__global__ void __launch_bounds__(D)
    paged_combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse,
                         bf16* __restrict__ out, int splits) {
  const int64_t row = blockIdx.x;
  const int d = threadIdx.x;
  const float* lse = ws_lse + row * splits;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, lse[s]);
  float den = 0.f, num = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      if (lse[s] == -INFINITY) continue;
      const float w = exp2f(lse[s] - mx);
      den += w;
      num += w * ws_o[(row * splits + s) * D + d];
    }
  }
  out[row * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

template <int D, int G>
int launch_g(const bf16* q, const bf16* k, const bf16* v, const int32_t* pt, const int32_t* cu,
             const int32_t* kl, bf16* out, float* ws_o, float* ws_lse, int N, int num_seqs,
             int max_pages, int Hq, int Hkv, int pps, int splits, float sl2, cudaStream_t s) {
  constexpr int SMEM = paged_smem_bytes<D, G>();
  static_assert(SMEM <= 227 * 1024, "paged attention shared memory");
  auto kern = paged_attn_kernel<D, G>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    configured = true;
  }
  kern<<<dim3(splits, Hkv, N), 128, SMEM, s>>>(q, k, v, pt, cu, kl, out, ws_o, ws_lse, num_seqs,
                                              max_pages, Hq, Hkv, pps, splits, sl2);
  if (splits > 1)
    paged_combine_kernel<D><<<N * Hq, D, 0, s>>>(ws_o, ws_lse, out, splits);
  return 0;
}

template <int D>
int launch_d(const bf16* q, const bf16* k, const bf16* v, const int32_t* pt, const int32_t* cu,
             const int32_t* kl, bf16* out, float* ws_o, float* ws_lse, int N, int num_seqs,
             int max_pages, int Hq, int Hkv, int pps, int splits, float sl2, cudaStream_t s) {
#define CFB_PAGED_G(GV)                                                                       \
  case GV:                                                                                    \
    return launch_g<D, GV>(q, k, v, pt, cu, kl, out, ws_o, ws_lse, N, num_seqs, max_pages, Hq, \
                           Hkv, pps, splits, sl2, s);
  switch (Hq / Hkv) {
    CFB_PAGED_G(1)
    CFB_PAGED_G(2)
    CFB_PAGED_G(4)
    CFB_PAGED_G(7)
    CFB_PAGED_G(8)
    default: return -3;
  }
#undef CFB_PAGED_G
}

// New tokens' projections into the paged cache, one warp per (token, head):
// kqv [N, (Hkv + Hq + Hkv) * D] holds each token's k | q | v heads.  q and k
// heads get RMSNorm over D (when qk_norm) and rotate-half RoPE at the token's
// position (cos/sin tables [P, D/2] fp32), in fp32 with one rounding; q goes to
// q_out [N, Hq, D], k and v straight into their pool slots [slot, Hkv, D].
template <int D>
__global__ void __launch_bounds__(256)
    paged_qkv_rope_kernel(const bf16* __restrict__ kqv, const bf16* __restrict__ qw,
                          const bf16* __restrict__ kw, const float* __restrict__ cos_t,
                          const float* __restrict__ sin_t, const int64_t* __restrict__ pos,
                          const int64_t* __restrict__ slots, bf16* __restrict__ q_out,
                          bf16* __restrict__ k_layer, bf16* __restrict__ v_layer, int N, int Hq,
                          int Hkv, float eps, int qk_norm) {
  constexpr int PL = D / 64;  // rotation pairs per lane: dims j and j + D/2
  const int Htot = Hq + 2 * Hkv;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (w >= static_cast<int64_t>(N) * Htot) return;
  const int t = static_cast<int>(w / Htot), h = static_cast<int>(w % Htot);
  const bf16* src = kqv + w * D;
  const int j0 = lane * PL;
  float a[PL], b[PL];
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    a[i] = __bfloat162float(src[j0 + i]);
    b[i] = __bfloat162float(src[j0 + i + D / 2]);
  }
  const int64_t slot = slots[t];
  if (h >= Hkv + Hq) {  // v head: copy into the pool
    bf16* dst = v_layer + (slot * Hkv + (h - Hkv - Hq)) * D;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      dst[j0 + i] = __float2bfloat16(a[i]);
      dst[j0 + i + D / 2] = __float2bfloat16(b[i]);
    }
    return;
  }
  const bool is_k = h < Hkv;
  if (qk_norm) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PL; ++i) ss += a[i] * a[i] + b[i] * b[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / D + eps);
    const bf16* nw = is_k ? kw : qw;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      a[i] *= r * __bfloat162float(nw[j0 + i]);
      b[i] *= r * __bfloat162float(nw[j0 + i + D / 2]);
    }
  }
  const int64_t p = pos[t];
  bf16* dst = is_k ? k_layer + (slot * Hkv + h) * D
                   : q_out + (static_cast<int64_t>(t) * Hq + (h - Hkv)) * D;
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const float c = cos_t[p * (D / 2) + j0 + i], sn = sin_t[p * (D / 2) + j0 + i];
    dst[j0 + i] = __float2bfloat16(a[i] * c - b[i] * sn);
    dst[j0 + i + D / 2] = __float2bfloat16(b[i] * c + a[i] * sn);
  }
}

}  // namespace

int paged_qkv_rope(const bf16* kqv, const bf16* qw, const bf16* kw, const float* cos_t,
                   const float* sin_t, const int64_t* pos, const int64_t* slots, bf16* q_out,
                   bf16* k_layer, bf16* v_layer, int N, int Hq, int Hkv, int D, float eps,
                   bool qk_norm, cudaStream_t s) {
  const int64_t warps = static_cast<int64_t>(N) * (Hq + 2 * Hkv);
  const int grid = static_cast<int>((warps + 7) / 8);
  if (N <= 0) return 0;
  if (D == 64)
    paged_qkv_rope_kernel<64><<<grid, 256, 0, s>>>(kqv, qw, kw, cos_t, sin_t, pos, slots, q_out,
                                                   k_layer, v_layer, N, Hq, Hkv, eps, qk_norm);
  else if (D == 128)
    paged_qkv_rope_kernel<128><<<grid, 256, 0, s>>>(kqv, qw, kw, cos_t, sin_t, pos, slots, q_out,
                                                    k_layer, v_layer, N, Hq, Hkv, eps, qk_norm);
  else
    return -2;
  return static_cast<int>(cudaGetLastError());
}

void paged_attention_split(int N, int Hkv, int max_kv, int num_sms, int* pages_per_split,
                           int* splits) {
  const int pages = max_kv > 0 ? (max_kv + kPage - 1) / kPage : 1;
  // enough CTAs for about eight per SM; every warp keeps at least two pages
  const int target = 8 * num_sms;
  int sp = (target + N * Hkv - 1) / (N * Hkv);
  const int most = (pages + 2 * kWarps - 1) / (2 * kWarps);
  if (sp > most) sp = most;
  if (sp < 1) sp = 1;
  int pps = (pages + sp - 1) / sp;
  pps = (pps + kWarps - 1) / kWarps * kWarps;
  *pages_per_split = pps;
  *splits = (pages + pps - 1) / pps;
}

int paged_attention(const bf16* q, const bf16* k_pool, const bf16* v_pool,
                    const int32_t* page_table, const int32_t* cu_q, const int32_t* kv_lens,
                    bf16* out, float* ws_o, float* ws_lse, int N, int num_seqs, int max_pages,
                    int Hq, int Hkv, int D, int page_size, int pages_per_split, int splits,
                    float scale, cudaStream_t s) {
  if (page_size != kPage) return -4;
  if (splits < 1 || pages_per_split < 1) return -5;
  if (splits > 1 && (ws_o == nullptr || ws_lse == nullptr)) return -6;
  if (static_cast<int64_t>(splits) * pages_per_split < max_pages) return -7;
  if (N > 65535 || Hkv > 65535 || splits > 65535) return -8;
  const float sl2 = scale * 1.4426950408889634f;
  int rc;
  if (D == 64)
    rc = launch_d<64>(q, k_pool, v_pool, page_table, cu_q, kv_lens, out, ws_o, ws_lse, N,
                      num_seqs, max_pages, Hq, Hkv, pages_per_split, splits, sl2, s);
  else if (D == 128)
    rc = launch_d<128>(q, k_pool, v_pool, page_table, cu_q, kv_lens, out, ws_o, ws_lse, N,
                       num_seqs, max_pages, Hq, Hkv, pages_per_split, splits, sl2, s);
  else
    return -2;
  if (rc) return rc;
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
