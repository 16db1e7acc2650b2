// Causal / full flash-attention backward for sm_100a on tcgen05 tensor cores.
//
// Given Q, K, V, the forward output O, its log-sum-exp and dO:
//   P    = exp(scale * Q K^T - LSE)          dV = P^T dO
//   dP   = dO V^T                            dS = P * (dP - rowsum(dO * O))
//   dQ   = scale * dS K                      dK = scale * dS^T Q
// GQA without K/V replication: the gradients of one K/V head sum over the
// Hq/Hkv query heads of its group inside one CTA, so dK/dV need no atomics.
//
// Three launches:
//   bwd_prep_k   Delta = rowsum(dO * O) and -LSE in the log2 domain into
//                [B*Hq, S_pad] buffers (padding rows: Delta 0, -LSE -inf), and
//                zero the fp32 dQ accumulator [B*Hq, S_pad, D].
//   flash_bwd_kernel  one CTA per (128-key tile, b, kv head).  K and V stay
//                resident in shared memory; the CTA walks every 64-query half
//                tile of every query head of the group (causal: only those at
//                or after the key tile).  Everything is computed transposed,
//                keys on the 128 TMEM lanes:
//                  S^T  = K Q^T, dP^T = V dO^T              (SS MMAs, N = 64)
//                  P^T, dS^T written back into TMEM as bf16 over S^T / dP^T
//                  dV  += P^T dO, dK += dS^T Q             (A operand in TMEM)
//                  dQ   = dS K  (head_dim 64: per pair of halves, M = 128 queries)
//                  dQ^T = K^T dS^T (head_dim 128: per half, M = 128 = head_dim)
//                dS^T also goes to shared memory (the B/A operand of the dQ
//                MMA); dQ tiles are added to the fp32 accumulator with TMA
//                bulk reduce-add from a 128B-swizzled staging tile.
//   bwd_post_k   dQ(bf16) = scale * accumulator, in the layout of Q.
//
// Warp roles of the main kernel (704 threads):
//   warps 0-3    dQ warpgroup: TMEM -> swizzled staging -> TMA reduce-add
//   warps 4-19   four softmax-gradient warpgroups: 4-11 take the even half tiles,
//                12-19 the odd ones; within a pair each warpgroup owns 32 of the
//                64 query columns (one key row per thread), with packed f32x2
//                math; afterwards they write dV (4-11) and dK (12-19)
//   warp 20      TMA producer: K, V once; Q/dO/LSE/Delta half tiles through a ring
//   warp 21      MMA issuer (one thread)
// For head_dim 64, S^T/dP^T are double-buffered in TMEM, so the tensor core
// computes the next half's S^T and dP^T while two warpgroups turn the previous
// one into P^T and dS^T.
//
// Reference counterpart: the autograd backward of F.scaled_dot_product_attention
// (complexity/core/attention/gqa.py:229-265) and of the Triton flash kernel in
// complexity_cuda/fused_attention.py:120-232.
#include "common.cuh"
#include "flash.h"

namespace cfb {
namespace {

constexpr int kKT = 128;  // keys per CTA (TMEM lanes)
constexpr int kQH = 64;   // queries per half tile (MMA N)
// warp roles (TMEM lane quarter = warp % 4): warps 0-3 dQ, then NSW softmax
// warpgroups, then the producer and MMA warps
constexpr int kSoftWarp0 = 4;
#ifndef CFB_FLASH_NSW
#define CFB_FLASH_NSW 2
#endif

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// byte offset of element (row, col) of a [rows x 64] bf16 block in 128B-swizzle layout
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
  const int unit = (col >> 3) ^ (row & 7);
  return static_cast<uint32_t>(row * 128 + unit * 16 + (col & 7) * 2);
}

template <int D>
struct BwdCfg {
  static constexpr int CH = D / 64;                     // 64-element swizzle chunks along D
  static constexpr int NBUF = D == 64 ? 2 : 1;          // S^T/dP^T TMEM buffers
  static constexpr bool PAIR = D == 64;                 // dQ per pair of halves (M = 128 q)
  static constexpr int QST = D == 64 ? 4 : 2;           // Q/dO ring stages (half tiles)
  static constexpr int KV_BYTES = kKT * D * 2;          // one of K, V
  static constexpr int QH_BYTES = kQH * D * 2;          // one of Q, dO half tile
  static constexpr int LD_BYTES = 2 * kQH * 4;          // LSE (log2) + Delta of a half tile
  static constexpr int TX_BYTES = 2 * QH_BYTES + LD_BYTES;
  static constexpr int DS_BYTES = kKT * kQH * 2;        // dS^T of one half tile (16 KB)
  static constexpr int NDS = PAIR ? 4 : 2;              // dS^T slots: 2 pairs / 2 halves
  static constexpr int STG_BYTES = 32768;               // dQ staging (fp32, 128B-swizzled)
  // every swizzled tile starts on a 1024-byte boundary: K, V, Q ring, dO ring, LSE/Delta
  // ring (QST * 512 bytes, a multiple of 1024), dS^T slots, staging, barriers
  static constexpr int SMEM = 2 * KV_BYTES + QST * (2 * QH_BYTES + LD_BYTES) + NDS * DS_BYTES +
                              STG_BYTES + 1024 /*align*/ + 512 /*barriers*/;
  static_assert((QST * LD_BYTES) % 1024 == 0, "LSE/Delta ring keeps the next tile aligned");
  static_assert(SMEM <= 232448, "flash backward shared memory over the 227 KB limit");
  // TMEM columns: NBUF x {S^T, dP^T} fp32 (64 + 64), one bf16 {P^T, dS^T} region
  // (32 + 32, read by the dV/dK MMAs), dV, dK, dQ
  static constexpr uint32_t T_PD = NBUF * 128;
  static constexpr uint32_t T_DV = T_PD + 64;
  static constexpr uint32_t T_DK = T_DV + D;
  static constexpr uint32_t T_DQ = T_DK + D;
  static_assert(T_DQ + 64 <= 512, "TMEM budget");
  // softmax-gradient warpgroups: NSW / 2 per half tile, each owning CW query columns
  static constexpr int NSW = CFB_FLASH_NSW;
  static constexpr int CW = 2 * kQH / NSW;
  static constexpr int PRODUCER_WARP = kSoftWarp0 + 4 * NSW;
  static constexpr int MMA_WARP = PRODUCER_WARP + 1;
  static constexpr int THREADS = 32 * (MMA_WARP + 1);
};

struct BwdBars {
  uint64_t kv_full;
  uint64_t q_full[4];
  uint64_t q_empty[4];
  uint64_t s_full[2];
  uint64_t s_consumed[2];
  uint64_t pd_free[2];
  uint64_t ds_ready[2];
  uint64_t ds_empty[4];
  uint64_t dq_full;
  uint64_t dq_empty;
  uint64_t dkv_full;
  uint64_t mma_done;
  uint32_t tmem;
  int abort;
  int dq_go;
};

struct BwdParams {
  int B, Hq, Hkv, S, S_pad;
  float scale, scale_log2;
  int causal;
  const float* lse2;    // [B*Hq, S_pad]
  const float* delta;   // [B*Hq, S_pad]
  __nv_bfloat16* dk;    // element (b, h, s, d) at b*k_sb + h*k_sh + s*k_ss + d
  __nv_bfloat16* dv;
  int64_t k_sb, k_sh, k_ss;
};

// Pipeline timeline for profiling builds only (CFB_FLASH_TRACE defined): SM clock
// stamps of each hand-off in CTA 0, event kind e and index i at g_trace[e][i].
#ifdef CFB_FLASH_TRACE
__device__ long long g_trace[16][512];
#define FLASH_TRACE(e, i) \
  do { if (blockIdx.x == 0 && (i) < 512) g_trace[e][i] = clock64(); } while (0)
#else
#define FLASH_TRACE(e, i) do { } while (0)
#endif

// bounded wait whose verdict is the same for every lane of the warp
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               volatile int* abort_flag, int* err, int code,
                                               int site) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err, code, site));
}

// bounded wait that ignores the abort flag (drains this CTA's own TMA loads / MMAs)
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t start = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - start > kWaitBoundNs) return;
}

template <int D>
__global__ void __launch_bounds__(BwdCfg<D>::THREADS, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                     const __grid_constant__ CUtensorMap tmDQ, const BwdParams p, int* err) {
  using Cfg = BwdCfg<D>;
  constexpr int CH = Cfg::CH;
  constexpr int NBUF = Cfg::NBUF;
  constexpr int QST = Cfg::QST;
  constexpr bool PAIR = Cfg::PAIR;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + Cfg::KV_BYTES;
  uint8_t* sQ = sV + Cfg::KV_BYTES;                          // QST half tiles
  uint8_t* sdO = sQ + QST * Cfg::QH_BYTES;                   // QST half tiles
  uint8_t* sLD = sdO + QST * Cfg::QH_BYTES;                  // QST x {-lse2[64], delta[64]}
  uint8_t* sDS = sLD + QST * Cfg::LD_BYTES;
  uint8_t* sStg = sDS + Cfg::NDS * Cfg::DS_BYTES;
  BwdBars* bars = reinterpret_cast<BwdBars*>(sStg + Cfg::STG_BYTES);
  volatile int* abort_flag = &bars->abort;
  auto stQ = [&](int st) { return sQ + st * Cfg::QH_BYTES; };
  auto stdO = [&](int st) { return sdO + st * Cfg::QH_BYTES; };
  auto stLse = [&](int st) { return reinterpret_cast<float*>(sLD + st * Cfg::LD_BYTES); };
  auto stDelta = [&](int st) { return stLse(st) + kQH; };
  // dS^T of half tile w lives in slot ds_slot(w): pairs (head_dim 64) use two
  // adjacent slots per dQ tile so the pair is one MN-major operand
  auto ds_slot = [&](int w) { return PAIR ? ((w >> 1) & 1) * 2 + (w & 1) : (w & 1); };

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int BG = p.B * p.Hkv;
  const int kt = static_cast<int>(blockIdx.x) / BG;          // heaviest key tiles first
  const int bg = static_cast<int>(blockIdx.x) % BG;
  const int b = bg / p.Hkv, g = bg % p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int k0 = kt * kKT;
  const int nh = p.S_pad / kQH;                              // half tiles per head
  const int t0 = p.causal ? k0 / kQH : 0;
  const int per_head = nh - t0;                              // even
  const int n_iter = G * per_head;

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(&bars->q_full[s], 1);
      mbar_init(&bars->q_empty[s], 1);
      mbar_init(&bars->ds_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_consumed[i], 4 * (Cfg::NSW / 2));  // the warps of one half
      mbar_init(&bars->pd_free[i], 1);
      mbar_init(&bars->ds_ready[i], 4 * (Cfg::NSW / 2));
    }
    mbar_init(&bars->dq_full, 1);
    mbar_init(&bars->dq_empty, 4);
    mbar_init(&bars->dkv_full, 1);
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
      mbar_arrive_expect_tx(&bars->kv_full, 2 * Cfg::KV_BYTES);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        tma_load_4d(sK + c * kKT * 128, &tmK, &bars->kv_full, c * 64, k0, g, b);
        tma_load_4d(sV + c * kKT * 128, &tmV, &bars->kv_full, c * 64, k0, g, b);
      }
      int issued = 0;
      for (int u = 0; u < n_iter; ++u) {
        const int st = u % QST;
        if (!mbar_wait(&bars->q_empty[st], ((u / QST) & 1) ^ 1, abort_flag, err, kErrTimeoutEmpty,
                       60))
          break;
        const int h = g * G + u / per_head;
        const int q0 = (t0 + u % per_head) * kQH;
        const int64_t row = (static_cast<int64_t>(b) * p.Hq + h) * p.S_pad + q0;
        FLASH_TRACE(0, u);
        mbar_arrive_expect_tx(&bars->q_full[st], Cfg::TX_BYTES);
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          tma_load_4d(stQ(st) + c * kQH * 128, &tmQ, &bars->q_full[st], c * 64, q0, h, b);
          tma_load_4d(stdO(st) + c * kQH * 128, &tmdO, &bars->q_full[st], c * 64, q0, h, b);
        }
        bulk_load(stLse(st), p.lse2 + row, kQH * 4, &bars->q_full[st]);
        bulk_load(stDelta(st), p.delta + row, kQH * 4, &bars->q_full[st]);
        ++issued;
      }
      // never leave the CTA with its own loads in flight
      drain_wait(&bars->kv_full, 0);
      for (int u = issued - QST < 0 ? 0 : issued - QST; u < issued; ++u)
        drain_wait(&bars->q_full[u % QST], (u / QST) & 1);
    }
  } else if (warp == Cfg::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC_S = idesc_bf16(kKT, kQH, false, false);   // S^T, dP^T
      constexpr uint32_t IDESC_G = idesc_bf16(kKT, D, false, true);      // dV, dK
      constexpr uint32_t IDESC_Q = idesc_bf16(128, PAIR ? D : kQH, true, true);  // dQ / dQ^T
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      bool ok = mbar_wait(&bars->kv_full, 0, abort_flag, err, kErrTimeoutFull, 61);
      // iteration v issues S^T/dP^T of half v (into buffer v % NBUF, once the
      // softmax of half v - NBUF has read that buffer), then dV/dK (and dQ) of
      // half v - NBUF once its P^T/dS^T are packed
      for (int v = 0; v < n_iter + NBUF && ok; ++v) {
        if (v < n_iter) {
          const int st = v % QST;
          if (!mbar_wait(&bars->q_full[st], (v / QST) & 1, abort_flag, err, kErrTimeoutFull, 62)) {
            ok = false;
            break;
          }
          if (v >= NBUF) {
            const int vp = v - NBUF;
            if (!mbar_wait(&bars->s_consumed[vp & 1], (vp >> 1) & 1, abort_flag, err,
                           kErrTimeoutTmem, 70)) {
              ok = false;
              break;
            }
          }
          tc_fence_after();
          const uint32_t tb = tmem + (v % NBUF) * 128;
          const uint32_t q_base = smem_u32(stQ(st)), do_base = smem_u32(stdO(st));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t ka = (kk >> 2) * (kKT * 128) + (kk & 3) * 32;
            const uint32_t kb = (kk >> 2) * (kQH * 128) + (kk & 3) * 32;
            umma_bf16(tb, sw128_desc(k_base + ka, 16, 1024), sw128_desc(q_base + kb, 16, 1024),
                      IDESC_S, kk != 0 ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t ka = (kk >> 2) * (kKT * 128) + (kk & 3) * 32;
            const uint32_t kb = (kk >> 2) * (kQH * 128) + (kk & 3) * 32;
            umma_bf16(tb + 64, sw128_desc(v_base + ka, 16, 1024),
                      sw128_desc(do_base + kb, 16, 1024), IDESC_S, kk != 0 ? 1u : 0u);
          }
          umma_commit(&bars->s_full[v & 1]);
          FLASH_TRACE(1, v);
        }
        const int w = v - NBUF;
        if (w < 0) continue;
        if (!mbar_wait(&bars->ds_ready[w & 1], (w >> 1) & 1, abort_flag, err, kErrTimeoutTmem,
                       63)) {
          ok = false;
          break;
        }
        tc_fence_after();
        FLASH_TRACE(2, w);
        const int st = w % QST;
        const uint32_t q_base = smem_u32(stQ(st)), do_base = smem_u32(stdO(st));
        // dV += P^T dO, dK += dS^T Q: A = the bf16 P^T / dS^T region of TMEM, B MN-major
#pragma unroll
        for (int kk = 0; kk < kQH / 16; ++kk)
          umma_bf16_ts(tmem + Cfg::T_DV, tmem + Cfg::T_PD + kk * 8,
                       sw128_desc(do_base + kk * 2048, kQH * 128, 1024), IDESC_G,
                       (w > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kQH / 16; ++kk)
          umma_bf16_ts(tmem + Cfg::T_DK, tmem + Cfg::T_PD + 32 + kk * 8,
                       sw128_desc(q_base + kk * 2048, kQH * 128, 1024), IDESC_G,
                       (w > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars->q_empty[st]);
        // the P^T/dS^T region is free for the next half (packed by the other warpgroups)
        umma_commit(&bars->pd_free[(w + 1) & 1]);
        if (PAIR && !(w & 1)) continue;
        const int n = PAIR ? (w >> 1) : w;       // dQ tile index
        if (!mbar_wait(&bars->dq_empty, (n & 1) ^ 1, abort_flag, err, kErrTimeoutTmem, 64)) {
          ok = false;
          break;
        }
        tc_fence_after();
        FLASH_TRACE(3, n);
        const int slot = n & 1;                  // ds_empty barrier of this dQ tile
        const uint32_t ds_base = smem_u32(sDS + ds_slot(PAIR ? w - 1 : w) * Cfg::DS_BYTES);
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk) {
          uint64_t ad, bd;
          if constexpr (PAIR) {
            // dQ[q, d] = dS[q, key] K[key, d]: A = dS (MN-major, 2 chunks of 64 q), B = K (MN-major)
            ad = sw128_desc(ds_base + kk * 2048, Cfg::DS_BYTES, 1024);
            bd = sw128_desc(k_base + kk * 2048, kKT * 128, 1024);
          } else {
            // dQ^T[d, q] = K^T[d, key] dS^T[key, q]: A = K^T (MN-major), B = dS^T (MN-major)
            ad = sw128_desc(k_base + kk * 2048, kKT * 128, 1024);
            bd = sw128_desc(ds_base + kk * 2048, Cfg::DS_BYTES, 1024);
          }
          umma_bf16(tmem + Cfg::T_DQ, ad, bd, IDESC_Q, kk != 0 ? 1u : 0u);
        }
        umma_commit(&bars->dq_full);
        umma_commit(&bars->ds_empty[slot]);
      }
      if (ok) umma_commit(&bars->dkv_full);
      // TMEM is freed only after every issued MMA has completed
      umma_commit(&bars->mma_done);
      drain_wait(&bars->mma_done, 0);
    }
  } else if (warp >= kSoftWarp0 && warp < Cfg::PRODUCER_WARP) {
    // ------------------- P^T / dS^T: one key row per thread, CW query columns
    constexpr int NPH = Cfg::NSW / 2;            // warpgroups per half tile
    constexpr int CW = Cfg::CW;
    const int sw = (warp - kSoftWarp0) >> 2;     // softmax warpgroup
    const int wg = sw / NPH;                     // halves w with w % 2 == wg
    const int cp = (sw % NPH) * CW;              // first query column of this warpgroup
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int kr = k0 + r;
    const bool key_ok = kr < p.S;
    const float2 sl2 = make_float2(p.scale_log2, p.scale_log2);
    bool ok = true;
    for (int w = wg; w < n_iter; w += 2) {
      const int it = w >> 1;
      const int st = w % QST;
      if (!mbar_wait_warp(&bars->s_full[wg], it & 1, abort_flag, err, kErrTimeoutTmem, 65) ||
          !mbar_wait_warp(&bars->q_full[st], (w / QST) & 1, abort_flag, err, kErrTimeoutFull, 66)) {
        ok = false;
        break;
      }
      const int n = PAIR ? (w >> 1) : w;         // dQ tile of this half
      const int slot = n & 1;
      uint8_t* ds_smem = sDS + ds_slot(w) * Cfg::DS_BYTES;
      if (!mbar_wait_warp(&bars->ds_empty[slot], ((n >> 1) & 1) ^ 1, abort_flag, err,
                          kErrTimeoutEmpty, 67)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (sw % NPH == 0 && threadIdx.x % 128 == 0) FLASH_TRACE(4, w);
      const int q0 = (t0 + w % per_head) * kQH;
      const uint32_t tb = tmem + lane_off + (w % NBUF) * 128 + cp;
      const float4* nl4 = reinterpret_cast<const float4*>(stLse(st) + cp);
      const float4* dl4 = reinterpret_cast<const float4*>(stDelta(st) + cp);
      const bool full = key_ok && (!p.causal || k0 + kKT - 1 <= q0 + cp) && (k0 + kKT <= p.S);
      uint32_t pk[CW / 2], dk[CW / 2];           // packed bf16 P^T and dS^T of this row
#pragma unroll
      for (int j = 0; j < CW / 16; ++j) {
        float s[16], dp[16];
        tmem_ld16(tb + 16 * j, s);
        tmem_ld16(tb + 64 + 16 * j, dp);
        tmem_wait_ld();
        if (j == CW / 16 - 1) {
          // S^T/dP^T are in registers: the tensor core may refill this buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->s_consumed[wg]);
        }
        if (sw == 0 && threadIdx.x % 128 == 0 && j < 2) FLASH_TRACE(8 + 3 * j, w);
        uint32_t* pkj = pk + 8 * j;
        uint32_t* dkj = dk + 8 * j;
        if (full) {
          // interior half: no masking; 16 elements as 8 packed pairs
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const float4 nl = nl4[4 * j + i4];   // -log2 LSE of 4 query columns
            const float4 dl = dl4[4 * j + i4];   // Delta of the same columns
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              const int i = 4 * i4 + 2 * h2;
              const float2 x = fma2(make_float2(s[i], s[i + 1]), sl2,
                                    h2 ? make_float2(nl.z, nl.w) : make_float2(nl.x, nl.y));
              const float2 pr = make_float2(ex2f(x.x), ex2f(x.y));
              const float2 dsv = mul2(pr, sub2(make_float2(dp[i], dp[i + 1]),
                                               h2 ? make_float2(dl.z, dl.w)
                                                  : make_float2(dl.x, dl.y)));
              pkj[i / 2] = pack_bf16x2(pr.x, pr.y);
              dkj[i / 2] = pack_bf16x2(dsv.x, dsv.y);
            }
          }
        } else {
          // diagonal / ragged half: causal and key-range masks
          const float* nl = stLse(st) + cp + 16 * j;
          const float* dl = stDelta(st) + cp + 16 * j;
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            float pr[2], dsv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int c = cp + 16 * j + i + e;  // query column within the half
              float pv = ex2f(fmaf(s[i + e], p.scale_log2, nl[i + e]));
              if (!key_ok || (p.causal && kr > q0 + c)) pv = 0.f;
              pr[e] = pv;
              dsv[e] = pv * (dp[i + e] - dl[i + e]);
            }
            pkj[i / 2] = pack_bf16x2(pr[0], pr[1]);
            dkj[i / 2] = pack_bf16x2(dsv[0], dsv[1]);
          }
        }
        if (sw == 0 && threadIdx.x % 128 == 0 && j < 2) FLASH_TRACE(9 + 3 * j, w);
        // dS^T for the dQ MMA (its own shared-memory slot)
#pragma unroll
        for (int u = 0; u < 2; ++u)
          *reinterpret_cast<uint4*>(ds_smem + sw128_off(r, cp + 16 * j + u * 8)) =
              make_uint4(dkj[4 * u], dkj[4 * u + 1], dkj[4 * u + 2], dkj[4 * u + 3]);
      }
      // the single P^T/dS^T region: wait until the dV/dK MMAs of half w - 1 have read it
      if (w >= 1 && !mbar_wait_warp(&bars->pd_free[wg], (((w + 1) >> 1) - 1) & 1, abort_flag,
                                    err, kErrTimeoutTmem, 71)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tpd = tmem + lane_off + Cfg::T_PD + cp / 2;
#pragma unroll
      for (int j = 0; j < CW / 16; ++j) {
        tmem_st8(tpd + 8 * j, pk + 8 * j);
        tmem_st8(tpd + 32 + 8 * j, dk + 8 * j);
      }
      tmem_wait_st();
      if (sw % NPH == 0 && threadIdx.x % 128 == 0) FLASH_TRACE(14, w);
      tc_fence_before();
      fence_proxy_async_shared();
      __syncwarp();
      if (sw % NPH == 0 && threadIdx.x % 128 == 0) FLASH_TRACE(5, w);
      if (lane == 0) mbar_arrive(&bars->ds_ready[wg]);
    }
    // ----------- dV (warpgroups 0, 1) / dK (2, 3), half of the head dim each
    if (ok && mbar_wait_warp(&bars->dkv_full, 0, abort_flag, err, kErrTimeoutTmem, 68)) {
      tc_fence_after();
      const bool is_dv = sw < NPH;
      const int c0 = (sw % NPH) * (D / NPH);
      const uint32_t col = (is_dv ? Cfg::T_DV : Cfg::T_DK) + c0;
      const float f = is_dv ? 1.f : p.scale;
      __nv_bfloat16* dst = (is_dv ? p.dv : p.dk) + b * p.k_sb + g * p.k_sh +
                           static_cast<int64_t>(kr) * p.k_ss + c0;
#pragma unroll
      for (int c = 0; c < D / NPH; c += 16) {
        float v[16];
        tmem_ld16(tmem + lane_off + col + c, v);
        tmem_wait_ld();
        if (key_ok) {
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            uint4 o;
            o.x = pack_bf16x2(v[8 * u] * f, v[8 * u + 1] * f);
            o.y = pack_bf16x2(v[8 * u + 2] * f, v[8 * u + 3] * f);
            o.z = pack_bf16x2(v[8 * u + 4] * f, v[8 * u + 5] * f);
            o.w = pack_bf16x2(v[8 * u + 6] * f, v[8 * u + 7] * f);
            *reinterpret_cast<uint4*>(dst + c + 8 * u) = o;
          }
        }
      }
    }
  } else {
    // ----------------------- dQ (warps 0-3): TMEM -> staging -> TMA reduce-add
    const int wq = warp & 3;
    const int lt = wq * 32 + lane;                 // TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool leader = threadIdx.x == 0;
    volatile int* go = &bars->dq_go;               // leader's verdict for this tile
    const int ndq = PAIR ? n_iter / 2 : n_iter;
    for (int n = 0; n < ndq; ++n) {
      // the leader alone waits (staging free, dQ tile ready) and tells the
      // warpgroup, so a timeout cannot leave threads behind at the named barrier
      if (leader) {
        bulk_wait_group_read<0>();
        *go = mbar_wait(&bars->dq_full, n & 1, abort_flag, err, kErrTimeoutTmem, 69) ? 1 : 0;
      }
      named_bar_sync(1, 128);
      if (!*go) break;
      tc_fence_after();
      if (leader) FLASH_TRACE(6, n);
      const int u = PAIR ? 2 * n : n;
      const int h = g * G + u / per_head;
      const int q0 = (t0 + u % per_head) * kQH;
      if constexpr (PAIR) {
        // lane = query row (128 rows), 64 d values: two boxes [128 rows][32 fp32]
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          float v[32];
          tmem_ld32(tmem + lane_off + Cfg::T_DQ + bx * 32, v);
          tmem_wait_ld();
          if (bx == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->dq_empty);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(sStg + bx * 16384 + lt * 128 + ((j ^ (lt & 7)) * 16)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      } else {
        // lane = d (128), 64 query values in two passes of 32: four boxes
        // [64 rows][32 fp32], box = lt / 32
        uint8_t* box = sStg + wq * 8192;
        const int dd = lt & 31;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float v[32];
          tmem_ld32(tmem + lane_off + Cfg::T_DQ + half * 32, v);
          tmem_wait_ld();
          if (half == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->dq_empty);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int q = half * 32 + i;
            *reinterpret_cast<float*>(box + q * 128 + ((((dd >> 2) ^ (q & 7)) * 16)) +
                                      (dd & 3) * 4) = v[i];
          }
        }
      }
      fence_proxy_async_shared();
      named_bar_sync(1, 128);
      if (leader) {
        const int row = (b * p.Hq + h) * p.S_pad + q0;
        constexpr int NBX = PAIR ? 2 : 4;
#pragma unroll
        for (int bx = 0; bx < NBX; ++bx)
          tma_reduce_add_2d(&tmDQ, sStg + bx * (PAIR ? 16384 : 8192), bx * 32, row);
        bulk_commit_group();
        FLASH_TRACE(7, n);
      }
    }
    if (leader) bulk_wait_group_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == Cfg::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Delta = rowsum(dO * O), LSE -> log2 domain, zero the dQ accumulator.
// D/8 threads per (b, h, s) row, 8 elements each.
template <int D>
__global__ void bwd_prep_k(Bhsd o, Bhsd dout, const float* __restrict__ lse, float* lse2,
                           float* delta, float* dqacc, int B, int Hq, int S, int S_pad) {
  constexpr int TPR = D / 8;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = gid / TPR;                   // (b*Hq + h)*S_pad + s
  const int part = static_cast<int>(gid % TPR);
  if (row >= static_cast<int64_t>(B) * Hq * S_pad) return;
  const int s = static_cast<int>(row % S_pad);
  const int bh = static_cast<int>(row / S_pad);
  const int b = bh / Hq, h = bh % Hq;
  float acc = 0.f;
  if (s < S) {
    const uint4 ov = *reinterpret_cast<const uint4*>(
        static_cast<const __nv_bfloat16*>(o.p) + b * o.sb + h * o.sh + s * o.ss + part * 8);
    const uint4 dv = *reinterpret_cast<const uint4*>(
        static_cast<const __nv_bfloat16*>(dout.p) + b * dout.sb + h * dout.sh + s * dout.ss +
        part * 8);
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&ov);
    const uint32_t* c = reinterpret_cast<const uint32_t*>(&dv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = unpack_bf16x2(a[i]), y = unpack_bf16x2(c[i]);
      acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
    }
  }
#pragma unroll
  for (int m = TPR / 2; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  float4* z = reinterpret_cast<float4*>(dqacc + row * D + part * 8);
  z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (part == 0) {
    delta[row] = acc;
    lse2[row] = s < S ? -lse[static_cast<int64_t>(bh) * S + s] * 1.4426950408889634f : -INFINITY;
  }
}

// dq = bf16(scale * accumulator), 8 elements per thread
template <int D>
__global__ void bwd_post_k(const float* __restrict__ dqacc, Bhsd dq, int B, int Hq, int S,
                           int S_pad, float scale) {
  constexpr int TPR = D / 8;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t r = gid / TPR;                     // (b*Hq + h)*S + s (valid rows only)
  const int part = static_cast<int>(gid % TPR);
  if (r >= static_cast<int64_t>(B) * Hq * S) return;
  const int s = static_cast<int>(r % S);
  const int bh = static_cast<int>(r / S);
  const int b = bh / Hq, h = bh % Hq;
  const float4* src =
      reinterpret_cast<const float4*>(dqacc + (static_cast<int64_t>(bh) * S_pad + s) * D + part * 8);
  const float4 x = src[0], y = src[1];
  uint4 o;
  o.x = pack_bf16x2(x.x * scale, x.y * scale);
  o.y = pack_bf16x2(x.z * scale, x.w * scale);
  o.z = pack_bf16x2(y.x * scale, y.y * scale);
  o.w = pack_bf16x2(y.z * scale, y.w * scale);
  *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dq.p) + b * dq.sb + h * dq.sh + s * dq.ss +
                            part * 8) = o;
}

template <int D>
int launch_bwd(const Bhsd& q, const Bhsd& k, const Bhsd& v, const Bhsd& o, const Bhsd& dout,
               const float* lse, const Bhsd& dq, const Bhsd& dk, const Bhsd& dv, int B, int Hq,
               int Hkv, int S, float scale, bool causal, float* work, cudaStream_t stream,
               int* err) {
  using Cfg = BwdCfg<D>;
  const int S_pad = flash_bwd_pad(S);
  const int64_t rows = static_cast<int64_t>(B) * Hq * S_pad;
  float* lse2 = work;
  float* delta = work + rows;
  float* dqacc = work + 2 * rows;
  CUtensorMap tq, tk, tv, tdo, tdq;
  int rc = make_bhsd_map(&tq, q, B, Hq, S, D, kQH);
  if (!rc) rc = make_bhsd_map(&tdo, dout, B, Hq, S, D, kQH);
  if (!rc) rc = make_bhsd_map(&tk, k, B, Hkv, S, D, kKT);
  if (!rc) rc = make_bhsd_map(&tv, v, B, Hkv, S, D, kKT);
  if (!rc) {
    const int64_t dims[2] = {D, rows};
    const int64_t strides[1] = {static_cast<int64_t>(D) * 4};
    const int box[2] = {32, Cfg::PAIR ? 128 : 64};
    rc = make_tmap_nd(&tdq, dqacc, 2, dims, strides, box, true, true);
  }
  if (rc) return rc;
  {
    const int64_t threads = rows * (D / 8);
    bwd_prep_k<D><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
        o, dout, lse, lse2, delta, dqacc, B, Hq, S, S_pad);
  }
  BwdParams prm;
  prm.B = B;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.S = S;
  prm.S_pad = S_pad;
  prm.scale = scale;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal ? 1 : 0;
  prm.lse2 = lse2;
  prm.delta = delta;
  prm.dk = static_cast<__nv_bfloat16*>(dk.p);
  prm.dv = static_cast<__nv_bfloat16*>(dv.p);
  prm.k_sb = dk.sb;
  prm.k_sh = dk.sh;
  prm.k_ss = dk.ss;
  if (dv.sb != dk.sb || dv.sh != dk.sh || dv.ss != dk.ss) return -4;
  auto kern = flash_bwd_kernel<D>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM))
    return static_cast<int>(cudaGetLastError());
  const dim3 grid((S_pad / kKT) * B * Hkv);
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(tq, tk, tv, tdo, tdq, prm, err);
  {
    const int64_t threads = static_cast<int64_t>(B) * Hq * S * (D / 8);
    bwd_post_k<D><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
        dqacc, dq, B, Hq, S, S_pad, scale);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

int make_bhsd_map(CUtensorMap* m, const Bhsd& t, int B, int H, int S, int D, int rows) {
  const int64_t dims[4] = {D, S, H, B};
  const int64_t strides[3] = {t.ss * 2, t.sh * 2, t.sb * 2};
  const int box[4] = {64, rows, 1, 1};
  return make_tmap_nd(m, t.p, 4, dims, strides, box, false, true);
}

int flash_bwd_pad(int S) { return (S + kKT - 1) / kKT * kKT; }

int64_t flash_bwd_workspace_floats(int B, int Hq, int S, int D) {
  const int64_t rows = static_cast<int64_t>(B) * Hq * flash_bwd_pad(S);
  return rows * (2 + D);
}

int flash_bwd_launch(const Bhsd& q, const Bhsd& k, const Bhsd& v, const Bhsd& o,
                     const Bhsd& dout, const float* lse, const Bhsd& dq, const Bhsd& dk,
                     const Bhsd& dv, int B, int Hq, int Hkv, int S, int D, float scale,
                     bool causal, float* workspace, cudaStream_t stream, int* err) {
  if (Hq % Hkv) return -3;
  if (D == 64)
    return launch_bwd<64>(q, k, v, o, dout, lse, dq, dk, dv, B, Hq, Hkv, S, scale, causal,
                          workspace, stream, err);
  if (D == 128)
    return launch_bwd<128>(q, k, v, o, dout, lse, dq, dk, dv, B, Hq, Hkv, S, scale, causal,
                           workspace, stream, err);
  return -2;
}

}  // namespace cfb
