// Causal / full flash-attention forward for sm_100a on tcgen05 tensor cores.
//
//   O[b, s, h, :] = softmax(scale * Q[b,h,s,:] K[b,g(h),:,:]^T) V[b,g(h),:,:]
//   LSE[b, h, s]  = log(sum_k exp(scale * q.k))          (for the backward)
//
// q: [B, Hq, S, D], k/v: [B, Hkv, S, D] (bf16, any strides along b, h, s with d
// contiguous: head-major, or the token-major q written by the QK-norm/RoPE
// kernel, read in place through 4-D TMA maps), GQA group g(h) = h / (Hq/Hkv)
// -- K/V are never replicated.  O is written token-major
// [B, S, Hq*D] so the o_proj GEMM reads it directly.  D in {64, 128}.
//
// One CTA per (NQ x 128 query rows, b*Hq); NQ = 2 for head_dim 64, 1 for 128.
// Warp roles:
//   warp 0      TMA producer: the NQ Q tiles once, then K_j/V_j through a ring
//   warp 1      MMA issuer (one thread): S_x(j) = Q_x K_j^T for every Q tile x,
//               then PV_x(j-1) = P_x(j-1) V_{j-1}, all accumulating in TMEM
//   warps 4..   one softmax warpgroup per Q tile, one query row per thread:
//               read S_x(j) from TMEM (two passes: max, then exp2), fold the
//               previous tile's PV into fp32 output registers with the running
//               rescale, write P_x(j) (bf16) to 128B-swizzled shared memory.
// The tensor cores compute S for one Q tile while the other tile's warpgroup
// is in softmax, and K/V tiles are shared by the NQ Q tiles.
// Reference counterpart: F.scaled_dot_product_attention after K/V
// repeat_interleave in complexity/core/attention/gqa.py:153-154,229-265.
#include "common.cuh"
#include "flash.h"

namespace cfb {
namespace {

constexpr int kQT = 128;   // query rows per Q tile
constexpr int kKT = 128;   // keys per KV tile

// 2^x on the SFU (hardware approximation, relative error ~2^-22)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
struct FlashCfg {
  // head_dim 64: two Q tiles per CTA share each K/V tile (two softmax warpgroups);
  // head_dim 128: one Q tile (shared memory holds fewer, larger tiles)
  static constexpr int NQ = D == 64 ? 2 : 1;
  static constexpr int STAGES = D == 64 ? 3 : 2;
  static constexpr int CHUNKS = D / 64;                 // 128-byte swizzle atoms along D
  static constexpr int Q_BYTES = kQT * D * 2;
  static constexpr int K_BYTES = kKT * D * 2;
  static constexpr int V_BYTES = kKT * D * 2;
  static constexpr int P_BYTES = kQT * kKT * 2;         // two 64-key chunks
  static constexpr int SMEM =
      NQ * Q_BYTES + STAGES * (K_BYTES + V_BYTES) + NQ * P_BYTES + 1024 + 512;
  static constexpr uint32_t TMEM_COLS = 512;            // S_x (128 each) then PV_x (D each)
  static constexpr int THREADS = 128 + 128 * NQ;
  static_assert(SMEM <= 232448, "flash forward shared memory over the 227 KB limit");
};

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[3];
  uint64_t kv_empty[3];
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
__global__ void __launch_bounds__(FlashCfg<D>::THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ out,
                     float* __restrict__ lse, int B, int Hq, int Hkv, int S, float scale_log2,
                     int causal, int* err) {
  using Cfg = FlashCfg<D>;
  constexpr int NQ = Cfg::NQ;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int CTA_Q = NQ * kQT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                                   // NQ tiles
  uint8_t* sK = sQ + NQ * Cfg::Q_BYTES;
  uint8_t* sV = sK + STAGES * Cfg::K_BYTES;
  uint8_t* sP = sV + STAGES * Cfg::V_BYTES;             // NQ tiles
  Bars* bars = reinterpret_cast<Bars*>(sP + NQ * Cfg::P_BYTES);
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
  const int nkv = causal ? min(nkv_all, (min(q0 + CTA_Q, S) - 1) / kKT + 1) : nkv_all;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < NQ; ++i) {
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      mbar_arrive_expect_tx(&bars->q_full, NQ * Cfg::Q_BYTES);
#pragma unroll
      for (int x = 0; x < NQ; ++x)
#pragma unroll
        for (int c = 0; c < Cfg::CHUNKS; ++c)
          tma_load_4d(sQ + x * Cfg::Q_BYTES + c * kQT * 128, &tmQ, &bars->q_full, c * 64,
                      q0 + x * kQT, h, b);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!mbar_wait(&bars->kv_empty[st], ph ^ 1, abort_flag, err, kErrTimeoutEmpty, 30)) break;
        mbar_arrive_expect_tx(&bars->kv_full[st], Cfg::K_BYTES + Cfg::V_BYTES);
#pragma unroll
        for (int c = 0; c < Cfg::CHUNKS; ++c) {
          tma_load_4d(sK + st * Cfg::K_BYTES + c * kKT * 128, &tmK, &bars->kv_full[st], c * 64,
                      j * kKT, g, b);
          tma_load_4d(sV + st * Cfg::V_BYTES + c * kKT * 128, &tmV, &bars->kv_full[st], c * 64,
                      j * kKT, g, b);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IDESC_S = idesc_bf16(kQT, kKT, false, false);
      constexpr uint32_t IDESC_PV = idesc_bf16(kQT, D, false, true);
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag, err, kErrTimeoutFull, 31);
      for (int j = 0; j <= nkv && ok; ++j) {
        const int st = j % STAGES;
        if (j < nkv) {
          if (!mbar_wait(&bars->kv_full[st], (j / STAGES) & 1, abort_flag, err, kErrTimeoutFull,
                         34)) {
            ok = false;
            break;
          }
          const uint32_t k_base = smem_u32(sK + st * Cfg::K_BYTES);
#pragma unroll
          for (int x = 0; x < NQ; ++x) {
            // S_x(j) overwrites S_x(j-1): wait until its softmax has read it
            if (!mbar_wait(&bars->s_empty[x], (j & 1) ^ 1, abort_flag, err, kErrTimeoutTmem, 35)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t q_base = smem_u32(sQ + x * Cfg::Q_BYTES);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * (kQT * 128) + (kk & 3) * 32;
              umma_bf16(tmem + x * 128, sw128_desc(q_base + off, 16, 1024),
                        sw128_desc(k_base + off, 16, 1024), IDESC_S, kk != 0 ? 1u : 0u);
            }
            umma_commit(&bars->s_full[x]);
          }
          if (!ok) break;
        }
        if (j > 0) {
          // PV_x(j-1) = P_x(j-1) V_{j-1}
          const int jp = j - 1;
          const int sp = jp % STAGES;
          const uint32_t v_base = smem_u32(sV + sp * Cfg::V_BYTES);
#pragma unroll
          for (int x = 0; x < NQ; ++x) {
            if (!mbar_wait(&bars->p_full[x], jp & 1, abort_flag, err, kErrTimeoutFull, 32) ||
                !mbar_wait(&bars->pv_empty[x], (jp & 1) ^ 1, abort_flag, err, kErrTimeoutTmem,
                           33)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t p_base = smem_u32(sP + x * Cfg::P_BYTES);
#pragma unroll
            for (int kk = 0; kk < kKT / 16; ++kk) {
              const uint64_t ad =
                  sw128_desc(p_base + (kk >> 2) * (kQT * 128) + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = sw128_desc(v_base + kk * 2048, kKT * 128, 1024);
              umma_bf16(tmem + NQ * 128 + x * D, ad, bd, IDESC_PV, kk != 0 ? 1u : 0u);
            }
            umma_commit(&bars->pv_full[x]);
          }
          if (!ok) break;
          umma_commit(&bars->kv_empty[sp]);  // K and V of tile j-1 are no longer needed
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ softmax + correction
    const int x = (warp - 4) >> 2;               // which Q tile this warpgroup owns
    const int wq = warp & 3;
    const int r = wq * 32 + lane;                 // query row within the tile
    const int qpos = q0 + x * kQT + r;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t t_s = tmem + x * 128 + lane_off;
    const uint32_t t_pv = tmem + NQ * 128 + x * D + lane_off;
    uint8_t* pt = sP + x * Cfg::P_BYTES;
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    float m = -INFINITY;      // running max (log2 domain)
    float l = 0.f;            // running sum
    float alpha_prev = 1.f;   // rescale owed to the output when PV_{j-1} is folded in
    bool ok = true;

    for (int j = 0; j < nkv && ok; ++j) {
      if (!mbar_wait(&bars->s_full[x], j & 1, abort_flag, err, kErrTimeoutTmem, 37)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * kKT;
      int kmax = S - k0;   // keys valid for this row: < S and (causal) <= qpos
      if (causal) kmax = min(kmax, qpos - k0 + 1);
      const bool full = kmax >= kKT;  // interior tile: no masking needed
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kKT; c += 32) {
        float v[32];
        tmem_ld32(t_s + c, v);
        tmem_wait_ld();
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c + i < kmax) mx = fmaxf(mx, v[i]);
        }
      }
      const float m_new = fmaxf(m, mx * scale_log2);
      const float alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
      const float msub = (m_new == -INFINITY) ? 0.f : m_new;
      // fold PV_{j-1} before P_j overwrites P_{j-1} in shared memory
      if (j > 0) {
        if (!mbar_wait(&bars->pv_full[x], (j - 1) & 1, abort_flag, err, kErrTimeoutTmem, 36)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          float v[32];
          tmem_ld32(t_pv + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c + i] = o[c + i] * alpha_prev + v[i];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->pv_empty[x]);
      }
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kKT; c += 32) {
        float v[32];
        tmem_ld32(t_s + c, v);
        tmem_wait_ld();
        uint32_t pk[16];
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = ex2(v[i] * scale_log2 - msub);
            const float p1 = ex2(v[i + 1] * scale_log2 - msub);
            rs += p0 + p1;
            pk[i / 2] = pack_bf16x2(p0, p1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = (c + i < kmax) ? ex2(v[i] * scale_log2 - msub) : 0.f;
            const float p1 = (c + i + 1 < kmax) ? ex2(v[i + 1] * scale_log2 - msub) : 0.f;
            rs += p0 + p1;
            pk[i / 2] = pack_bf16x2(p0, p1);
          }
        }
        uint8_t* chunk = pt + (c >> 6) * (kQT * 128);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(chunk + sw128_off(r, (c & 63) + u * 8)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      }
      // S_j has been read: the MMA warp may overwrite this buffer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_empty[x]);
      // P_j visible to the tensor core (async proxy) before signalling
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[x]);
      l = l * alpha + rs;
      m = m_new;
      alpha_prev = alpha;
    }
    if (ok && nkv > 0) {
      const int jl = nkv - 1;
      if (mbar_wait(&bars->pv_full[x], jl & 1, abort_flag, err, kErrTimeoutTmem, 38)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          float v[32];
          tmem_ld32(t_pv + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c + i] = o[c + i] * alpha_prev + v[i];
        }
      }
    }
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
            l > 0.f ? (m + __log2f(l)) * 0.69314718055994531f : -INFINITY;
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
  if (D == 64) {
    using Cfg = FlashCfg<64>;
    auto kern = flash_fwd_kernel<64>;
    const dim3 grid(((S + Cfg::NQ * kQT - 1) / (Cfg::NQ * kQT)) * B * Hq);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM))
      return static_cast<int>(cudaGetLastError());
    kern<<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(tq, tk, tv, static_cast<__nv_bfloat16*>(out),
                                                    lse, B, Hq, Hkv, S, sl2, causal ? 1 : 0, err);
  } else {
    using Cfg = FlashCfg<128>;
    auto kern = flash_fwd_kernel<128>;
    const dim3 grid(((S + Cfg::NQ * kQT - 1) / (Cfg::NQ * kQT)) * B * Hq);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM))
      return static_cast<int>(cudaGetLastError());
    kern<<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(tq, tk, tv, static_cast<__nv_bfloat16*>(out),
                                                    lse, B, Hq, Hkv, S, sl2, causal ? 1 : 0, err);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace cfb
