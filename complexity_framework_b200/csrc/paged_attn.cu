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
//   three-stage cp.async ring in shared memory: the next two pages' K/V
//   (2 x 4 KB each) are in flight while the current one is consumed.  K rows are padded by 16
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
  static constexpr int ROW = D * 2 + 16;               // bytes per K or V row, padded
  static constexpr int K_BYTES = kPage * ROW;
  static constexpr int STAGE = 2 * K_BYTES;            // K page then V page
  static constexpr int NSTAGE = 3;                     // pages in flight per warp: 2
  static constexpr int WARP = NSTAGE * STAGE;
  static constexpr int RING = kWarps * WARP;
};

template <int D, int G>
constexpr int paged_smem_bytes() {
  // ring (reused for the warp merge: kWarps x G x D fp32) + (m, l) per warp and head
  return (PagedSmem<D>::RING > kWarps * G * D * 4 ? PagedSmem<D>::RING : kWarps * G * D * 4) +
         2 * kWarps * G * 4;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
// d += a (16x16 bf16, row) * b (16x8 bf16, col), fp32 accumulators
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Per page (16 keys) and warp, on 16x8x16 bf16 tensor-core fragments: the G
// query heads of this KV head are the rows of a 16-row tile (rows >= G are
// zero), S = Q K^T is two 16x8 tiles (keys 0-7, 8-15) over D/16 k-steps with
// K fragments from ldmatrix; the online softmax runs on the accumulator
// fragments (lane owns rows lane/4 and lane/4+8, keys 2(lane%4)+{0,1} of each
// tile); P re-packs in registers into the A operand of O += P V, whose V
// fragments come from ldmatrix.trans.  This keeps the instruction count per
// page near 200, so the loop is bound by HBM rather than by issue.
template <int D, int G>
__global__ void __launch_bounds__(128)
    paged_attn_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k_pool,
                      const bf16* __restrict__ v_pool, const int32_t* __restrict__ page_table,
                      const int32_t* __restrict__ cu_q, const int32_t* __restrict__ kv_lens,
                      bf16* __restrict__ out, float* __restrict__ ws_o,
                      float* __restrict__ ws_lse, int num_seqs, int max_pages, int Hq, int Hkv,
                      int pages_per_split, int splits, float scale_log2) {
  static_assert(G <= 16, "one 16-row tile of query heads");
  using S = PagedSmem<D>;
  constexpr int KS = D / 16;          // k-steps of Q K^T
  constexpr int NT = D / 8;           // n-tiles of O
  constexpr int CHUNKS = D * 2 / 16;  // 16-byte chunks per K or V row
  constexpr int MERGE = S::RING > kWarps * G * D * 4 ? S::RING : kWarps * G * D * 4;
  extern __shared__ __align__(128) uint8_t smem[];
  float* s_m = reinterpret_cast<float*>(smem + MERGE);            // [kWarps][G]
  float* s_l = s_m + kWarps * G;                                  // [kWarps][G]

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int tok = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int lo = 0, hi = num_seqs - 1;  // sequence of this token (binary search over cu_q)
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

  // ---- this warp's pages: p_begin + warp + kWarps * i, through a 3-stage ring
  const int first = p_begin + warp;
  const int count = first < p_end ? (p_end - first + kWarps - 1) / kWarps : 0;
  uint8_t* ring = smem + warp * S::WARP;
  auto issue = [&](int i) {
    const int page = __ldg(pt + first + kWarps * i);
    uint8_t* st = ring + (i % S::NSTAGE) * S::STAGE;
    const int64_t base = (static_cast<int64_t>(page) * kPage * Hkv + kvh) * D;
#pragma unroll
    for (int c = lane; c < kPage * CHUNKS; c += 32) {
      const int r = c / CHUNKS, x = c % CHUNKS;
      const int64_t g = base + static_cast<int64_t>(r) * Hkv * D + x * 8;
      cp_async16(st + r * S::ROW + x * 16, k_pool + g);
      cp_async16(st + S::K_BYTES + r * S::ROW + x * 16, v_pool + g);
    }
  };
#pragma unroll
  for (int j = 0; j < S::NSTAGE - 1; ++j) {  // one commit group per ring slot, even if empty
    if (j < count) issue(j);
    cp_async_commit();
  }

  // ---- Q as A fragments: rows = heads (>= G are zero), one 16x16 tile per k-step
  const int fr = lane >> 2, fc = (lane & 3) * 2;
  uint32_t qa[KS][4];
  {
    const bf16* q0 = q + orow * D;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int c0 = ks * 16 + fc;
      auto ld2 = [&](int row, int col) -> uint32_t {
        if (row >= G) return 0u;
        return *reinterpret_cast<const uint32_t*>(q0 + row * D + col);
      };
      qa[ks][0] = ld2(fr, c0);
      qa[ks][1] = ld2(fr + 8, c0);
      qa[ks][2] = ld2(fr, c0 + 8);
      qa[ks][3] = ld2(fr + 8, c0 + 8);
    }
  }
  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows fr, fr + 8
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
  // ldmatrix row addresses: lane supplies row (lane & 7) of matrix (lane >> 3)
  const int lm = lane >> 3, lr = lane & 7;

  for (int i = 0; i < count; ++i) {
    if (i + S::NSTAGE - 1 < count) issue(i + S::NSTAGE - 1);
    cp_async_commit();
    cp_async_wait<S::NSTAGE - 1>();  // page i has landed
    __syncwarp();
    const int slot = i % S::NSTAGE;
    const uint32_t st = ring_s + slot * S::STAGE;
    const int p = first + kWarps * i;
    const int nk = min(kPage, n_keys - p * kPage);
    if (nk < kPage) {  // partial last page: zero the unwritten V rows (P is 0 there)
      uint8_t* vs = ring + slot * S::STAGE + S::K_BYTES;
      for (int c = lane; c < (kPage - nk) * CHUNKS; c += 32)
        *reinterpret_cast<uint4*>(vs + (nk + c / CHUNKS) * S::ROW + (c % CHUNKS) * 16) =
            make_uint4(0, 0, 0, 0);
      __syncwarp();
    }
    // ---- S = Q K^T: tile 0 = keys 0-7, tile 1 = keys 8-15
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      // matrices: (keys 0-7, dims +0), (keys 0-7, +8), (keys 8-15, +0), (keys 8-15, +8)
      const uint32_t addr = st + ((lm >> 1) * 8 + lr) * S::ROW + (ks * 16 + (lm & 1) * 8) * 2;
      uint32_t b00, b01, b10, b11;
      ldsm_x4(addr, b00, b01, b10, b11);
      mma16816(s0, qa[ks], b00, b01);
      mma16816(s1, qa[ks], b10, b11);
    }
    // ---- online softmax on the fragments (exp2 domain), masked past n_keys
    const int k0 = fc, k1 = fc + 1, k2 = 8 + fc, k3 = 9 + fc;
    s0[0] = k0 < nk ? s0[0] * scale_log2 : -INFINITY;
    s0[1] = k1 < nk ? s0[1] * scale_log2 : -INFINITY;
    s0[2] = k0 < nk ? s0[2] * scale_log2 : -INFINITY;
    s0[3] = k1 < nk ? s0[3] * scale_log2 : -INFINITY;
    s1[0] = k2 < nk ? s1[0] * scale_log2 : -INFINITY;
    s1[1] = k3 < nk ? s1[1] * scale_log2 : -INFINITY;
    s1[2] = k2 < nk ? s1[2] * scale_log2 : -INFINITY;
    s1[3] = k3 < nk ? s1[3] * scale_log2 : -INFINITY;
    float mx0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
    float mx1 = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: key 0 is valid
    const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);  // exp2(-inf) = 0 on the first page
    m0 = mn0;
    m1 = mn1;
    float p0[4], p1[4];
    p0[0] = exp2f(s0[0] - mn0);
    p0[1] = exp2f(s0[1] - mn0);
    p0[2] = exp2f(s0[2] - mn1);
    p0[3] = exp2f(s0[3] - mn1);
    p1[0] = exp2f(s1[0] - mn0);
    p1[1] = exp2f(s1[1] - mn0);
    p1[2] = exp2f(s1[2] - mn1);
    p1[3] = exp2f(s1[3] - mn1);
    l0 = l0 * a0 + (p0[0] + p0[1] + p1[0] + p1[1]);  // lane-partial row sums
    l1 = l1 * a1 + (p0[2] + p0[3] + p1[2] + p1[3]);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      o[j][0] *= a0;
      o[j][1] *= a0;
      o[j][2] *= a1;
      o[j][3] *= a1;
    }
    // ---- O += P V: P as the A fragment (rows = heads, k = the page's 16 keys)
    uint32_t pa[4] = {pack2_bf16(p0[0], p0[1]), pack2_bf16(p0[2], p0[3]),
                      pack2_bf16(p1[0], p1[1]), pack2_bf16(p1[2], p1[3])};
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      // matrices (trans): (keys 0-7, dims j*8), (keys 8-15, j*8), (keys 0-7, j*8+8), (8-15, +8)
      const uint32_t addr =
          st + S::K_BYTES + ((lm & 1) * 8 + lr) * S::ROW + (j * 8 + (lm >> 1) * 8) * 2;
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(addr, v0, v1, v2, v3);
      mma16816(o[j], pa, v0, v1);
      mma16816(o[j + 1], pa, v2, v3);
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
  }
  cp_async_wait<0>();
  // full row sums across the quad
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // ---- merge the warps (the ring is free now): rows < G only
  __syncthreads();
  float* s_acc = reinterpret_cast<float*>(smem);  // [kWarps][G][D]
  if ((lane & 3) == 0) {
    if (fr < G) {
      s_m[warp * G + fr] = m0;
      s_l[warp * G + fr] = l0;
    }
    if (fr + 8 < G) {
      s_m[warp * G + fr + 8] = m1;
      s_l[warp * G + fr + 8] = l1;
    }
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int d = j * 8 + fc;
    if (fr < G) {
      s_acc[(warp * G + fr) * D + d] = o[j][0];
      s_acc[(warp * G + fr) * D + d + 1] = o[j][1];
    }
    if (fr + 8 < G) {
      s_acc[(warp * G + fr + 8) * D + d] = o[j][2];
      s_acc[(warp * G + fr + 8) * D + d + 1] = o[j][3];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float mm = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, s_m[w * G + g]);
    float ll = 0.f, acc = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float mw = s_m[w * G + g];
      if (mw == -INFINITY) continue;  // a warp without pages
      const float f = exp2f(mw - mm);
      ll += s_l[w * G + g] * f;
      acc += s_acc[(w * G + g) * D + d] * f;
    }
    const float val = ll > 0.f ? acc / ll : 0.f;
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
