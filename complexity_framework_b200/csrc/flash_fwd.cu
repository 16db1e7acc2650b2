// Causal / full flash-attention forward for sm_100a on tcgen05 tensor cores.
//
//   O[b, s, h, :] = softmax(scale * Q[b,h,s,:] K[b,g(h),:,:]^T) V[b,g(h),:,:]
//   LSE[b, h, s]  = log(sum_k exp(scale * q.k))          (for the backward)
//
// q: [B, Hq, S, D], k/v: [B, Hkv, S, D] (head-major, bf16), GQA group g(h) =
// h / (Hq/Hkv) -- K/V are never replicated.  O is written token-major
// [B, S, Hq*D] so the o_proj GEMM reads it directly.  D in {64, 128}.
//
// One CTA per (128-query tile, b*Hq).  Warp roles:
//   warp 0    TMA producer: Q once, then K_j/V_j tiles through a 3-stage ring
//   warp 1    MMA issuer (one thread): S_j = Q K_j^T into TMEM (double
//             buffered), then PV_{j-1} = P_{j-1} V_{j-1} into TMEM (double buffered)
//   warps 4-7 softmax + correction, one query row per thread: read S_j from
//             TMEM, online max/sum in the exp2 domain, write P_j (bf16) to
//             128B-swizzled shared memory for the next MMA, then fold PV_{j-1}
//             into the fp32 output registers with the running rescale factor.
// So QK^T of tile j+1 runs on the tensor cores while tile j is in softmax.
// Reference counterpart: F.scaled_dot_product_attention after K/V
// repeat_interleave in complexity/core/attention/gqa.py:153-154,229-265.
#include "common.cuh"
#include "flash.h"

namespace cfb {
namespace {

constexpr int kQT = 128;   // query rows per CTA
constexpr int kKT = 128;   // keys per KV tile
constexpr int kStages = 3;

template <int D>
struct FlashCfg {
  static constexpr int CHUNKS = D / 64;                 // 128-byte swizzle atoms along D
  static constexpr int Q_BYTES = kQT * D * 2;
  static constexpr int K_BYTES = kKT * D * 2;
  static constexpr int V_BYTES = kKT * D * 2;
  static constexpr int P_BYTES = kQT * kKT * 2;         // two 64-key chunks
  static constexpr int SMEM = Q_BYTES + kStages * (K_BYTES + V_BYTES) + 2 * P_BYTES + 1024 + 512;
  static constexpr uint32_t TMEM_COLS = 512;            // S0 S1 (128 each) PV0 PV1 (D each)
};

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t p_full[2];
  uint64_t pv_full[2];
  uint64_t pv_empty[2];
  uint32_t tmem;
  int abort;
};

// byte offset of element (row, col) of a [rows x 64] bf16 block in 128B-swizzle layout
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
  const int unit = (col >> 3) ^ (row & 7);
  return static_cast<uint32_t>(row * 128 + unit * 16 + (col & 7) * 2);
}

template <int D>
__global__ void __launch_bounds__(256, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ out,
                     float* __restrict__ lse, int B, int Hq, int Hkv, int S, float scale_log2,
                     int causal, int* err) {
  using Cfg = FlashCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::Q_BYTES;
  uint8_t* sV = sK + kStages * Cfg::K_BYTES;
  uint8_t* sP = sV + kStages * Cfg::V_BYTES;
  Bars* bars = reinterpret_cast<Bars*>(sP + 2 * Cfg::P_BYTES);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int nqt = (S + kQT - 1) / kQT;
  const int BH = B * Hq;
  // heaviest (last) query tiles first so the tail of the grid is short work
  const int qt = nqt - 1 - static_cast<int>(blockIdx.x) / BH;
  const int bh = static_cast<int>(blockIdx.x) % BH;
  const int b = bh / Hq, h = bh % Hq;
  const int g = h / (Hq / Hkv);
  const int q0 = qt * kQT;
  const int nkv_all = (S + kKT - 1) / kKT;
  const int nkv = causal ? min(nkv_all, (q0 + kQT - 1) / kKT + 1) : nkv_all;
  const int q_row0 = (b * Hq + h) * S + q0;        // row in the [B*Hq*S, D] view
  const int kv_row0 = (b * Hkv + g) * S;           // row of key 0 in the [B*Hkv*S, D] view

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_empty[i], 4);
      mbar_init(&bars->p_full[i], 4);
      mbar_init(&bars->pv_full[i], 1);
      mbar_init(&bars->pv_empty[i], 4);
    }
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  const uint32_t t_s[2] = {tmem, tmem + 128};
  const uint32_t t_pv[2] = {tmem + 256, tmem + 256 + D};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      mbar_arrive_expect_tx(&bars->q_full, Cfg::Q_BYTES);
#pragma unroll
      for (int c = 0; c < Cfg::CHUNKS; ++c)
        tma_load_2d(sQ + c * kQT * 128, &tmQ, &bars->q_full, c * 64, q_row0);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(&bars->kv_empty[st], ph ^ 1, abort_flag, err, kErrTimeoutEmpty, 30)) break;
        mbar_arrive_expect_tx(&bars->kv_full[st], Cfg::K_BYTES + Cfg::V_BYTES);
#pragma unroll
        for (int c = 0; c < Cfg::CHUNKS; ++c) {
          tma_load_2d(sK + st * Cfg::K_BYTES + c * kKT * 128, &tmK, &bars->kv_full[st], c * 64,
                      kv_row0 + j * kKT);
          tma_load_2d(sV + st * Cfg::V_BYTES + c * kKT * 128, &tmV, &bars->kv_full[st], c * 64,
                      kv_row0 + j * kKT);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC_S = idesc_bf16(kQT, kKT, false, false);
      constexpr uint32_t IDESC_PV = idesc_bf16(kQT, D, false, true);
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag, err, kErrTimeoutFull, 31);
      const uint32_t q_base = smem_u32(sQ);
      auto issue_pv = [&](int j) -> bool {
        const int pb = j & 1;
        const int st = j % kStages;
        if (!mbar_wait(&bars->p_full[pb], (j >> 1) & 1, abort_flag, err, kErrTimeoutFull, 32))
          return false;
        if (!mbar_wait(&bars->pv_empty[pb], ((j >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutTmem,
                       33))
          return false;
        tc_fence_after();
        const uint32_t p_base = smem_u32(sP + pb * Cfg::P_BYTES);
        const uint32_t v_base = smem_u32(sV + st * Cfg::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk) {
          const uint64_t ad = sw128_desc(p_base + (kk >> 2) * (kQT * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(v_base + kk * 2048, kKT * 128, 1024);
          umma_bf16(t_pv[pb], ad, bd, IDESC_PV, kk != 0 ? 1u : 0u);
        }
        umma_commit(&bars->pv_full[pb]);
        umma_commit(&bars->kv_empty[st]);  // K_j and V_j no longer needed
        return true;
      };
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j % kStages;
        const int sb = j & 1;
        if (!mbar_wait(&bars->kv_full[st], (j / kStages) & 1, abort_flag, err, kErrTimeoutFull, 34) ||
            !mbar_wait(&bars->s_empty[sb], ((j >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutTmem,
                       35)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + st * Cfg::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kQT * 128) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kKT * 128) + (kk & 3) * 32;
          umma_bf16(t_s[sb], sw128_desc(q_base + off, 16, 1024), sw128_desc(k_base + koff, 16, 1024),
                    IDESC_S, kk != 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[sb]);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nkv > 0) issue_pv(nkv - 1);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ softmax + correction
    const int wq = warp & 3;
    const int r = wq * 32 + lane;                 // query row within the tile
    const int qpos = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    float m = -INFINITY;      // running max (log2 domain)
    float l = 0.f;            // running sum
    float alpha_prev = 1.f;   // rescale owed to the output when PV_{j-1} is folded in
    bool ok = true;

    auto fold_pv = [&](int j, float alpha) -> bool {
      const int pb = j & 1;
      if (!mbar_wait(&bars->pv_full[pb], (j >> 1) & 1, abort_flag, err, kErrTimeoutTmem, 36))
        return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float v[32];
        tmem_ld32(t_pv[pb] + lane_off + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c + i] = o[c + i] * alpha + v[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->pv_empty[pb]);
      return true;
    };

    for (int j = 0; j < nkv && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&bars->s_full[sb], (j >> 1) & 1, abort_flag, err, kErrTimeoutTmem, 37)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * kKT;
      // keys valid for this row: < S and (causal) <= qpos
      int kmax = S - k0;
      if (causal) kmax = min(kmax, qpos - k0 + 1);
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kKT; c += 32) {
        float v[32];
        tmem_ld32(t_s[sb] + lane_off + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c + i < kmax) mx = fmaxf(mx, v[i]);
      }
      const float m_new = fmaxf(m, mx * scale_log2);
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
      const float msub = (m_new == -INFINITY) ? 0.f : m_new;
      // pass 2: probabilities -> bf16 P tile (swizzled) and row sum
      float rs = 0.f;
      uint8_t* pt = sP + sb * Cfg::P_BYTES;
#pragma unroll
      for (int c = 0; c < kKT; c += 32) {
        float v[32];
        tmem_ld32(t_s[sb] + lane_off + c, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = (c + i < kmax) ? exp2f(v[i] * scale_log2 - msub) : 0.f;
          const float p1 = (c + i + 1 < kmax) ? exp2f(v[i + 1] * scale_log2 - msub) : 0.f;
          // the sum uses the bf16-rounded values the PV product will see
          const uint32_t w = pack_bf16x2(p0, p1);
          const float2 back = unpack_bf16x2(w);
          rs += back.x + back.y;
          pk[i / 2] = w;
        }
        uint8_t* chunk = pt + (c >> 6) * (kQT * 128);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int col = (c & 63) + u * 8;
          *reinterpret_cast<uint4*>(chunk + sw128_off(r, col)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      // S_j has been read: the MMA warp may overwrite this buffer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_empty[sb]);
      // P_j visible to the tensor core (async proxy) before signalling
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[sb]);
      l = l * alpha + rs;
      m = m_new;
      // fold PV_{j-1} (computed with max m_{j-1}) while the tensor cores work on PV_j
      if (j > 0 && !fold_pv(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && nkv > 0) ok = fold_pv(nkv - 1, alpha_prev);
    if (qpos < S) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (static_cast<int64_t>(b) * S + qpos) * Hq * D + h * D;
#pragma unroll
      for (int c = 0; c < D; c += 8) {
        uint4 w;
        w.x = pack_bf16x2(o[c] * inv, o[c + 1] * inv);
        w.y = pack_bf16x2(o[c + 2] * inv, o[c + 3] * inv);
        w.z = pack_bf16x2(o[c + 4] * inv, o[c + 5] * inv);
        w.w = pack_bf16x2(o[c + 6] * inv, o[c + 7] * inv);
        *reinterpret_cast<uint4*>(orow + c) = w;
      }
      if (lse != nullptr)
        lse[(static_cast<int64_t>(b) * Hq + h) * S + qpos] =
            l > 0.f ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace

int flash_fwd_launch(const void* q, const void* k, const void* v, void* out, float* lse, int B,
                     int Hq, int Hkv, int S, int D, float scale, bool causal, cudaStream_t stream,
                     int* err) {
  if (D != 64 && D != 128) return -2;
  if (Hq % Hkv) return -3;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, q, static_cast<int64_t>(B) * Hq * S, D, D, 64, kQT);
  if (!rc) rc = make_tmap_2d(&tk, k, static_cast<int64_t>(B) * Hkv * S, D, D, 64, kKT);
  if (!rc) rc = make_tmap_2d(&tv, v, static_cast<int64_t>(B) * Hkv * S, D, D, 64, kKT);
  if (rc) return rc;
  const int nqt = (S + kQT - 1) / kQT;
  const dim3 grid(nqt * B * Hq);
  const float sl2 = scale * 1.4426950408889634f;
  if (D == 64) {
    auto kern = flash_fwd_kernel<64>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FlashCfg<64>::SMEM);
    kern<<<grid, 256, FlashCfg<64>::SMEM, stream>>>(tq, tk, tv,
                                                    static_cast<__nv_bfloat16*>(out), lse, B, Hq,
                                                    Hkv, S, sl2, causal ? 1 : 0, err);
  } else {
    auto kern = flash_fwd_kernel<128>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FlashCfg<128>::SMEM);
    kern<<<grid, 256, FlashCfg<128>::SMEM, stream>>>(tq, tk, tv,
                                                     static_cast<__nv_bfloat16*>(out), lse, B, Hq,
                                                     Hkv, S, sl2, causal ? 1 : 0, err);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
