// Causal / full flash-attention forward for sm_100a on tcgen05 tensor cores.
//
//   O[b, s, h, :] = softmax(scale * Q[b,h,s,:] K[b,g(h),:,:]^T) V[b,g(h),:,:]
//   LSE[b, h, s]  = log(sum_k exp(scale * q.k))          (for the backward)
//
// q: [B, Hq, S, D], k/v: [B, Hkv, S, D] (bf16, any strides along b, h, s with d
// contiguous: head-major, or the token-major q written by the QK-norm/RoPE
// kernel, read in place through 4-D TMA maps), GQA group g(h) = h / (Hq/Hkv)
// -- K/V are never replicated.  O is written token-major [B, S, Hq*D] so the
// o_proj GEMM reads it directly.  D in {64, 128}.
//
// One CTA per (2 x 128 query rows, b*Hq): the two query tiles share every K/V
// tile.  TMEM holds, per query tile x, S_x (128 fp32 columns) and the output
// accumulator O_x (D columns); the bf16 probabilities P_x are packed in place
// over S_x and feed the P V MMA as its TMEM A operand, so P never goes through
// shared memory and O never through registers until the end.
// Warp roles (320 threads):
//   warps 0-3 / 4-7  softmax of query tile 0 / 1, one row per thread: the row
//                    of S is read from TMEM once (128 registers), its max taken,
//                    exponentials computed (a fixed share of them by a cubic on
//                    the FMA pipe, the rest on MUFU), P packed back into TMEM
//   warp 8           TMA producer: Q once, then K_j/V_j through a ring
//   warp 9           MMA issuer: per KV tile j and query tile x,
//                    O_x += P_x(j-1) V_{j-1}, then S_x(j) = Q_x K_j^T
// The running max is applied lazily: O and the row sum are rescaled only when
// the max grows by more than 2^8 (log2 units), which keeps P <= 256 (exact in
// bf16's exponent range) and makes rescaling rare after the first KV tiles.
// Rescaling needs no extra wait: S_x(j) is issued after O_x += P_x(j-1) V, so
// its completion implies that the accumulation reading O_x is done.
// Reference counterpart: F.scaled_dot_product_attention after K/V
// repeat_interleave in complexity/core/attention/gqa.py:153-154,229-265.
#include "common.cuh"
#include "flash.h"

namespace cfb {
namespace {

constexpr int kQT = 128;   // query rows per Q tile
constexpr int kKT = 128;   // keys per KV tile
constexpr int kNQ = 2;     // Q tiles per CTA
constexpr float kRescaleLog2 = 8.f;  // lazy-rescale threshold (log2 units)

#ifndef CFB_FLASH_FWD_POLY
#define CFB_FLASH_FWD_POLY 2  // of every 8 element pairs, this many use the cubic
#endif

// 2^x on the SFU (hardware approximation, relative error ~2^-22)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
struct FlashCfg {
  static constexpr int STAGES = D == 64 ? 4 : 2;
  static constexpr int CHUNKS = D / 64;                 // 128-byte swizzle atoms along D
  static constexpr int Q_BYTES = kQT * D * 2;
  static constexpr int K_BYTES = kKT * D * 2;
  static constexpr int V_BYTES = kKT * D * 2;
  static constexpr int SMEM = kNQ * Q_BYTES + STAGES * (K_BYTES + V_BYTES) + 1024 + 512;
  static constexpr uint32_t T_O = kNQ * 128;            // O_x at T_O + x * D
  static_assert(T_O + kNQ * D <= 512, "TMEM budget");
  static constexpr int PRODUCER_WARP = 8;
  static constexpr int MMA_WARP = 9;
  static constexpr int THREADS = 320;
  static_assert(SMEM <= 232448, "flash forward shared memory over the 227 KB limit");
};

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[4];
  uint64_t kv_empty[4];
  uint64_t s_full[kNQ];
  uint64_t p_full[kNQ];
  uint64_t o_full[kNQ];
  uint64_t mma_done;
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t start = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - start > kWaitBoundNs) return;
}

__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               volatile int* abort_flag, int* err, int code,
                                               int site) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err, code, site));
}

// 32 lanes x 32 columns store
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  tmem_st16(taddr, r);
  tmem_st16(taddr + 16, r + 16);
}

template <int D>
__global__ void __launch_bounds__(FlashCfg<D>::THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ out,
                     float* __restrict__ lse, int B, int Hq, int Hkv, int S, float scale_log2,
                     int causal, int* err) {
  using Cfg = FlashCfg<D>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int CTA_Q = kNQ * kQT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                                   // kNQ tiles
  uint8_t* sK = sQ + kNQ * Cfg::Q_BYTES;
  uint8_t* sV = sK + STAGES * Cfg::K_BYTES;
  Bars* bars = reinterpret_cast<Bars*>(sV + STAGES * Cfg::V_BYTES);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int nqt = (S + CTA_Q - 1) / CTA_Q;
  const int BH = B * Hq;
  // heaviest (last) query tiles first so the tail of the grid is short work
  const int qt = nqt - 1 - static_cast<int>(blockIdx.x) / BH;
  const int bh = static_cast<int>(blockIdx.x) % BH;
  const int b = bh / Hq, h = bh % Hq;
  const int g = h / (Hq / Hkv);
  const int q0 = qt * CTA_Q;
  const int nkv_all = (S + kKT - 1) / kKT;
  // KV tiles each query tile needs (causal: up to its last row)
  auto nkv_of = [&](int x) {
    return causal ? min(nkv_all, (min(q0 + (x + 1) * kQT, S) - 1) / kKT + 1) : nkv_all;
  };
  const int nkv = max(nkv_of(0), nkv_of(1));

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int x = 0; x < kNQ; ++x) {
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->p_full[x], 4);
      mbar_init(&bars->o_full[x], 1);
    }
    mbar_init(&bars->mma_done, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == Cfg::MMA_WARP) tmem_alloc(&bars->tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == Cfg::PRODUCER_WARP) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      mbar_arrive_expect_tx(&bars->q_full, kNQ * Cfg::Q_BYTES);
#pragma unroll
      for (int x = 0; x < kNQ; ++x)
#pragma unroll
        for (int c = 0; c < Cfg::CHUNKS; ++c)
          tma_load_4d(sQ + x * Cfg::Q_BYTES + c * kQT * 128, &tmQ, &bars->q_full, c * 64,
                      q0 + x * kQT, h, b);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int st = j % STAGES;
        if (!mbar_wait(&bars->kv_empty[st], ((j / STAGES) & 1) ^ 1, abort_flag, err,
                       kErrTimeoutEmpty, 30))
          break;
        mbar_arrive_expect_tx(&bars->kv_full[st], Cfg::K_BYTES + Cfg::V_BYTES);
#pragma unroll
        for (int c = 0; c < Cfg::CHUNKS; ++c) {
          tma_load_4d(sK + st * Cfg::K_BYTES + c * kKT * 128, &tmK, &bars->kv_full[st], c * 64,
                      j * kKT, g, b);
          tma_load_4d(sV + st * Cfg::V_BYTES + c * kKT * 128, &tmV, &bars->kv_full[st], c * 64,
                      j * kKT, g, b);
        }
        ++issued;
      }
      drain_wait(&bars->q_full, 0);
      for (int j = issued - STAGES < 0 ? 0 : issued - STAGES; j < issued; ++j)
        drain_wait(&bars->kv_full[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == Cfg::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC_S = idesc_bf16(kQT, kKT, false, false);
      constexpr uint32_t IDESC_PV = idesc_bf16(kQT, D, false, true);
      const int nkv_x[kNQ] = {nkv_of(0), nkv_of(1)};
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag, err, kErrTimeoutFull, 31);
      // O_x += P_x(jp) V_jp, A = the bf16 P_x packed over S_x in TMEM
      auto issue_pv = [&](int x, int jp) -> bool {
        if (!mbar_wait(&bars->p_full[x], jp & 1, abort_flag, err, kErrTimeoutFull, 32))
          return false;
        tc_fence_after();
        const uint32_t v_base = smem_u32(sV + (jp % STAGES) * Cfg::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk)
          umma_bf16_ts(tmem + Cfg::T_O + x * D, tmem + x * 128 + kk * 8,
                       sw128_desc(v_base + kk * 2048, kKT * 128, 1024), IDESC_PV,
                       (jp > 0 || kk > 0) ? 1u : 0u);
        return true;
      };
      for (int j = 0; j <= nkv && ok; ++j) {
        const int st = j % STAGES;
        if (j < nkv &&
            !mbar_wait(&bars->kv_full[st], (j / STAGES) & 1, abort_flag, err, kErrTimeoutFull,
                       34)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + st * Cfg::K_BYTES);
#pragma unroll
        for (int x = 0; x < kNQ; ++x) {
          if (j > 0 && j - 1 < nkv_x[x]) {
            if (!issue_pv(x, j - 1)) {
              ok = false;
              break;
            }
            if (j - 1 == nkv_x[x] - 1) umma_commit(&bars->o_full[x]);  // last accumulation
          }
          if (j < nkv_x[x]) {
            // S_x(j) = Q_x K_j^T (after O_x += P_x(j-1) V: S_x holds P_x until then)
            const uint32_t q_base = smem_u32(sQ + x * Cfg::Q_BYTES);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * (kQT * 128) + (kk & 3) * 32;
              umma_bf16(tmem + x * 128, sw128_desc(q_base + off, 16, 1024),
                        sw128_desc(k_base + off, 16, 1024), IDESC_S, kk != 0 ? 1u : 0u);
            }
            umma_commit(&bars->s_full[x]);
          }
        }
        if (!ok) break;
        if (j > 0) umma_commit(&bars->kv_empty[(j - 1) % STAGES]);  // K/V of tile j-1 done
      }
      umma_commit(&bars->mma_done);
      drain_wait(&bars->mma_done, 0);
    }
  } else if (warp < 4 * kNQ) {
    // ------------------------------------------------------------ softmax
    const int x = warp >> 2;                     // which Q tile this warpgroup owns
    const int wq = warp & 3;
    const int r = wq * 32 + lane;                 // query row within the tile
    const int qpos = q0 + x * kQT + r;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t t_s = tmem + x * 128 + lane_off;
    const uint32_t t_o = tmem + Cfg::T_O + x * D + lane_off;
    const int nkv_mine = nkv_of(x);
    float m_used = -INFINITY;  // max the current exponentials are relative to (log2 units)
    float l = 0.f;             // running sum of exponentials
    const float2 sl2 = make_float2(scale_log2, scale_log2);
    bool ok = true;

    for (int j = 0; j < nkv_mine && ok; ++j) {
      if (!mbar_wait_warp(&bars->s_full[x], j & 1, abort_flag, err, kErrTimeoutTmem, 37)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kKT];
#pragma unroll
      for (int c = 0; c < kKT; c += 32) tmem_ld32(t_s + c, s + c);
      tmem_wait_ld();
      const int k0 = j * kKT;
      int kmax = S - k0;   // keys valid for this row: < S and (causal) <= qpos
      if (causal) kmax = min(kmax, qpos - k0 + 1);
      if (kmax < kKT) {
#pragma unroll
        for (int c = 0; c < kKT; ++c)
          if (c >= kmax) s[c] = -INFINITY;
      }
      // row max over 8 independent partial maxima (a serial chain would cost
      // 128 dependent instructions of latency)
      float mp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mp[i] = s[i];
#pragma unroll
      for (int c = 8; c < kKT; ++c) mp[c & 7] = fmaxf(mp[c & 7], s[c]);
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      const float m_new = fmaxf(m_used, mx * scale_log2);
      // lazy rescale: only when the max grew by more than 2^kRescaleLog2
      const bool grow = m_new > m_used + kRescaleLog2;
      if (__any_sync(0xffffffffu, grow && m_used != -INFINITY)) {
        // O_x already holds P V of earlier tiles (their MMAs completed before S_x(j))
        const float alpha = (grow && m_used != -INFINITY) ? ex2(m_used - m_new) : 1.f;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          float o[32];
          uint32_t u[32];
          tmem_ld32(t_o + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(o[i] * alpha);
          tmem_st32(t_o + c, u);
        }
        tmem_wait_st();
      }
      if (grow) {
        if (m_used != -INFINITY) l *= ex2(m_used - m_new);
        m_used = m_new;
      }
      // rows with no valid key so far: every exponential is 0
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      const float2 nm = make_float2(-msub, -msub);
      float2 rs2[4] = {};                        // four independent partial row sums
#pragma unroll
      for (int c = 0; c < kKT; c += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 xv = fma2(make_float2(s[c + i], s[c + i + 1]), sl2, nm);
          const float2 pv = ((i >> 1) % 8) < CFB_FLASH_FWD_POLY
                                ? exp2_poly2(xv)
                                : make_float2(ex2(xv.x), ex2(xv.y));
          rs2[(i >> 1) & 3] = add2(rs2[(i >> 1) & 3], pv);
          pk[i / 2] = pack_bf16x2(pv.x, pv.y);
        }
        tmem_st16(t_s + c / 2, pk);              // bf16 P over already-read S columns
      }
      l += ((rs2[0].x + rs2[0].y) + (rs2[1].x + rs2[1].y)) +
           ((rs2[2].x + rs2[2].y) + (rs2[3].x + rs2[3].y));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[x]);
    }
    if (ok && nkv_mine > 0 &&
        mbar_wait_warp(&bars->o_full[x], 0, abort_flag, err, kErrTimeoutTmem, 38)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (static_cast<int64_t>(b) * S + qpos) * Hq * D + h * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(t_o + c, o);
        tmem_wait_ld();
        if (qpos < S) {
#pragma unroll
          for (int u = 0; u < 32; u += 8) {
            uint4 w;
            w.x = pack_bf16x2(o[u] * inv, o[u + 1] * inv);
            w.y = pack_bf16x2(o[u + 2] * inv, o[u + 3] * inv);
            w.z = pack_bf16x2(o[u + 4] * inv, o[u + 5] * inv);
            w.w = pack_bf16x2(o[u + 6] * inv, o[u + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c + u) = w;
          }
        }
      }
      if (qpos < S && lse != nullptr)
        lse[(static_cast<int64_t>(b) * Hq + h) * S + qpos] =
            l > 0.f ? (m_used + __log2f(l)) * 0.69314718055994531f : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == Cfg::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, void* out,
               float* lse, int B, int Hq, int Hkv, int S, float sl2, bool causal,
               cudaStream_t stream, int* err) {
  using Cfg = FlashCfg<D>;
  auto kern = flash_fwd_kernel<D>;
  const dim3 grid(((S + kNQ * kQT - 1) / (kNQ * kQT)) * B * Hq);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM))
    return static_cast<int>(cudaGetLastError());
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(tq, tk, tv, static_cast<__nv_bfloat16*>(out),
                                                  lse, B, Hq, Hkv, S, sl2, causal ? 1 : 0, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

int flash_fwd_launch(const Bhsd& q, const Bhsd& k, const Bhsd& v, void* out, float* lse, int B,
                     int Hq, int Hkv, int S, int D, float scale, bool causal, cudaStream_t stream,
                     int* err) {
  if (D != 64 && D != 128) return -2;
  if (Hq % Hkv) return -3;
  CUtensorMap tq, tk, tv;
  int rc = make_bhsd_map(&tq, q, B, Hq, S, D, kQT);
  if (!rc) rc = make_bhsd_map(&tk, k, B, Hkv, S, D, kKT);
  if (!rc) rc = make_bhsd_map(&tv, v, B, Hkv, S, D, kKT);
  if (rc) return rc;
  const float sl2 = scale * 1.4426950408889634f;
  return D == 64 ? launch_fwd<64>(tq, tk, tv, out, lse, B, Hq, Hkv, S, sl2, causal, stream, err)
                 : launch_fwd<128>(tq, tk, tv, out, lse, B, Hq, Hkv, S, sl2, causal, stream, err);
}

}  // namespace cfb
