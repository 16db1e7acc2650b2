// Memory-bound kernels of the TR-Hash decoder: RMSNorm fwd/bwd, fused
// QK-RMSNorm + RoPE + head-major scatter fwd/bwd, embedding fwd/bwd,
// cross-entropy loss+gradient from GEMM-epilogue partial statistics,
// deterministic-route expert scales, and the flat fp32-master AdamW.
//
// Reference counterparts: Liger RMSNorm/RoPE/FLCE used by
// complexity/core/normalization/norms.py:47-57, core/position/rotary.py:257-297,
// core/losses/fused_ce.py:95-204; routed weights of tr_hash/engine.py:66-104;
// torch.optim.AdamW as configured by training/trainer.py:329-334.
//
// All kernels use 16-byte vector accesses (8 bf16) and warp-per-row layouts;
// none uses scratch memory beyond its outputs.
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace cfb {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const bf16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z),
         d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ void store8(bf16* p, const float* v) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ float rb(float x) { return __bfloat162float(__float2bfloat16(x)); }

inline int grid_for(int64_t work, int per_block, int cap = 148 * 16) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

// ----------------------------------------------------------------- RMSNorm
__global__ void rmsnorm_fwd_k(const bf16* __restrict__ x, const bf16* __restrict__ w,
                              bf16* __restrict__ y, float* __restrict__ rstd, int64_t T, int H,
                              float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nv = H >> 3;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < T;
       row += warps) {
    const bf16* xr = x + row * H;
    float ss = 0.f;
    for (int i = lane; i < nv; i += 32) {
      float v[8];
      load8(xr + i * 8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / H + eps);
    for (int i = lane; i < nv; i += 32) {
      float v[8], wv[8];
      load8(xr + i * 8, v);
      load8(w + i * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = rb(v[j] * r) * wv[j];
      store8(y + row * H + i * 8, v);
    }
    if (lane == 0) rstd[row] = r;
  }
}

__global__ void rmsnorm_bwd_k(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                              const bf16* __restrict__ w, const float* __restrict__ rstd,
                              const bf16* __restrict__ dres, bf16* __restrict__ dx,
                              float* __restrict__ dw, int64_t T, int H) {
  extern __shared__ float sdw[];
  for (int i = threadIdx.x; i < H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nv = H >> 3;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < T;
       row += warps) {
    const float r = rstd[row];
    const bf16* xr = x + row * H;
    const bf16* dyr = dy + row * H;
    float dot = 0.f;
    for (int i = lane; i < nv; i += 32) {
      float xv[8], gv[8], wv[8];
      load8(xr + i * 8, xv);
      load8(dyr + i * 8, gv);
      load8(w + i * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        dot += gv[j] * wv[j] * xv[j];
        atomicAdd(&sdw[i * 8 + j], gv[j] * rb(xv[j] * r));
      }
    }
    dot = warp_sum(dot);
    const float c = dot * r * r * r / H;
    for (int i = lane; i < nv; i += 32) {
      float xv[8], gv[8], wv[8], o[8];
      load8(xr + i * 8, xv);
      load8(dyr + i * 8, gv);
      load8(w + i * 8, wv);
      if (dres != nullptr) {
        load8(dres + row * H + i * 8, o);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] += r * gv[j] * wv[j] - xv[j] * c;
      store8(dx + row * H + i * 8, o);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

// Register-accumulating variant for H <= NV*256: lane l owns vectors l, l+32, ...
// so its d(weight) partials live in registers for the whole row loop.  The
// weight row sits in shared memory and the second pass re-reads x / dy
// (L1-resident, just loaded) instead of holding them, which keeps the kernel
// near 64 registers so three 256-thread blocks fit per SM.
template <int NV>
__global__ void __launch_bounds__(256, 3)
    rmsnorm_bwd_reg_k(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                      const bf16* __restrict__ w, const float* __restrict__ rstd,
                      const bf16* __restrict__ dres, bf16* __restrict__ dx,
                      float* __restrict__ dw, int64_t T, int H) {
  extern __shared__ float sdw[];   // [H] d(weight) partials, then [H] weights
  float* sw = sdw + H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    sdw[i] = 0.f;
    sw[i] = __bfloat162float(w[i]);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nv = H >> 3;
  float acc[NV][8];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < T;
       row += warps) {
    const float r = rstd[row];
    const bf16* xr = x + row * H;
    const bf16* gr = dy + row * H;
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < nv) {
        float xv[8], gv[8];
        load8(xr + i * 8, xv);
        load8(gr + i * 8, gv);
        const float4 w0 = *reinterpret_cast<const float4*>(sw + i * 8);
        const float4 w1 = *reinterpret_cast<const float4*>(sw + i * 8 + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          dot += gv[j] * wv[j] * xv[j];
          acc[k][j] += gv[j] * rb(xv[j] * r);
        }
      }
    }
    dot = warp_sum(dot);
    const float c = dot * r * r * r / H;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < nv) {
        float xv[8], gv[8], o[8];
        load8(xr + i * 8, xv);
        load8(gr + i * 8, gv);
        if (dres != nullptr) {
          load8(dres + row * H + i * 8, o);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = 0.f;
        }
        const float4 w0 = *reinterpret_cast<const float4*>(sw + i * 8);
        const float4 w1 = *reinterpret_cast<const float4*>(sw + i * 8 + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += r * gv[j] * wv[j] - xv[j] * c;
        store8(dx + row * H + i * 8, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = lane + 32 * k;
    if (i < nv) {
#pragma unroll
      for (int j = 0; j < 8; ++j) atomicAdd(&sdw[i * 8 + j], acc[k][j]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

// ------------------------------------------------------- QK-norm + RoPE
// LPH = D/8 lanes cooperate on one (token, head) item with 16-byte vectors
// (lane gl of a group owns elements 8*gl .. 8*gl+7); a warp handles 32/LPH
// consecutive items of the flattened [token, head] order.  Head index hh:
// [0,Hq) q heads, [Hq, Hq+Hkv) k heads, [Hq+Hkv, Hq+2Hkv) v heads; the fused
// projection output kqv stores columns in k | q | v order.  The rotate-half
// partner of element j (j +- D/2) lives in lane gl ^ (LPH/2) of the group.
struct HeadItem {
  int64_t t;
  int hh;
  int col;
  int64_t hm;  // element offset of (b, head, s, 0) in the head-major tensor
  int kind;    // 0 = q, 1 = k, 2 = v
};

template <int D>
__device__ __forceinline__ HeadItem decode_item(int64_t item, int Htot, int S, int Hq, int Hkv,
                                                bool q_tm) {
  // item < 2^31 (checked by the launcher): 32-bit divisions are far cheaper
  HeadItem it;
  const uint32_t i32 = static_cast<uint32_t>(item);
  const uint32_t t32 = i32 / static_cast<uint32_t>(Htot);
  it.t = t32;
  it.hh = static_cast<int>(i32 - t32 * static_cast<uint32_t>(Htot));
  const int b = static_cast<int>(t32 / static_cast<uint32_t>(S));
  const int s = static_cast<int>(t32 - static_cast<uint32_t>(b) * static_cast<uint32_t>(S));
  if (it.hh < Hq) {
    it.kind = 0;
    it.col = Hkv * D + it.hh * D;
    // q is head-major [B, Hq, S, D], or token-major [B, S, Hq, D] with q_tm
    it.hm = q_tm ? (((int64_t)b * S + s) * Hq + it.hh) * D
                 : (((int64_t)b * Hq + it.hh) * S + s) * D;
  } else if (it.hh < Hq + Hkv) {
    const int h = it.hh - Hq;
    it.kind = 1;
    it.col = h * D;
    it.hm = (((int64_t)b * Hkv + h) * S + s) * D;
  } else {
    const int h = it.hh - Hq - Hkv;
    it.kind = 2;
    it.col = (Hkv + Hq) * D + h * D;
    it.hm = (((int64_t)b * Hkv + h) * S + s) * D;
  }
  return it;
}

__device__ __forceinline__ int s_of(int64_t t, int S) {
  return static_cast<int>(static_cast<uint32_t>(t) % static_cast<uint32_t>(S));
}

template <int LPH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8f(const float* p, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <int D>
__global__ void qk_norm_rope_fwd_k(const bf16* __restrict__ kqv, const bf16* __restrict__ qw,
                                   const bf16* __restrict__ kw, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const int32_t* __restrict__ pos,
                                   bf16* __restrict__ q, bf16* __restrict__ k,
                                   bf16* __restrict__ v, float* __restrict__ rstd, int B, int S,
                                   int Hq, int Hkv, float eps, bool qk_norm, bool q_tm) {
  constexpr int LPH = D / 8, GPW = 32 / LPH, HALF = LPH / 2;
  const int lane = threadIdx.x & 31;
  const int grp = lane / LPH, gl = lane % LPH;
  const int Htot = Hq + 2 * Hkv;
  const int C = Htot * D;
  const int64_t total = (int64_t)B * S * Htot;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t base = wid * GPW; base < total; base += nw * GPW) {
    const int64_t item = base + grp;
    const bool valid = item < total;
    HeadItem it = decode_item<D>(valid ? item : total - 1, Htot, S, Hq, Hkv, q_tm);
    float x[8];
    load8(kqv + it.t * C + it.col + gl * 8, x);
    const bool qk = it.kind != 2;
    if (qk_norm) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
      ss = group_sum<LPH>(ss);
      const float r = rsqrtf(ss / D + eps);
      if (qk) {
        float wv[8];
        load8((it.kind == 0 ? qw : kw) + gl * 8, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = rb(rb(x[j] * r) * wv[j]);
        if (gl == 0 && valid) rstd[it.t * (Hq + Hkv) + it.hh] = r;
      }
    }
    const int p = pos != nullptr ? pos[it.t] : s_of(it.t, S);
    float c[8], sn[8], o[8];
    load8f(cos_t + (int64_t)p * (D / 2) + (gl % HALF) * 8, c);
    load8f(sin_t + (int64_t)p * (D / 2) + (gl % HALF) * 8, sn);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[j], HALF);
      o[j] = gl < HALF ? x[j] * c[j] - partner * sn[j] : x[j] * c[j] + partner * sn[j];
      if (!qk) o[j] = x[j];
    }
    if (valid) {
      bf16* dst = it.kind == 0 ? q : (it.kind == 1 ? k : v);
      store8(dst + it.hm + gl * 8, o);
    }
  }
}

template <int D>
__global__ void __launch_bounds__(256, 3) qk_norm_rope_bwd_k(const bf16* __restrict__ dq, const bf16* __restrict__ dk,
                                   const bf16* __restrict__ dv, const bf16* __restrict__ kqv,
                                   const bf16* __restrict__ qw, const bf16* __restrict__ kw,
                                   const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                   const int32_t* __restrict__ pos, const float* __restrict__ rstd,
                                   bf16* __restrict__ dkqv, float* __restrict__ dqw,
                                   float* __restrict__ dkw, int B, int S, int Hq, int Hkv,
                                   bool qk_norm, bool q_tm) {
  constexpr int LPH = D / 8, GPW = 32 / LPH, HALF = LPH / 2;
  __shared__ float s_dqw[D], s_dkw[D];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    s_dqw[i] = 0.f;
    s_dkw[i] = 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int grp = lane / LPH, gl = lane % LPH;
  const int Htot = Hq + 2 * Hkv;
  const int C = Htot * D;
  const int64_t total = (int64_t)B * S * Htot;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  float accq[8], acck[8], wq[8], wk[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) accq[j] = acck[j] = 0.f;
  load8(qw + gl * 8, wq);
  load8(kw + gl * 8, wk);
  for (int64_t base = wid * GPW; base < total; base += nw * GPW) {
    const int64_t item = base + grp;
    const bool valid = item < total;
    HeadItem it = decode_item<D>(valid ? item : total - 1, Htot, S, Hq, Hkv, q_tm);
    const bf16* src = it.kind == 0 ? dq : (it.kind == 1 ? dk : dv);
    float g[8];
    load8(src + it.hm + gl * 8, g);
    const bool qk = it.kind != 2;
    // inverse rotation: dn_j = g_j cos_j + (first half ? g_{j+D/2} : -g_{j-D/2}) sin_j
    const int p = pos != nullptr ? pos[it.t] : s_of(it.t, S);
    float c[8], sn[8], dn[8];
    load8f(cos_t + (int64_t)p * (D / 2) + (gl % HALF) * 8, c);
    load8f(sin_t + (int64_t)p * (D / 2) + (gl % HALF) * 8, sn);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float partner = __shfl_xor_sync(0xffffffffu, g[j], HALF);
      dn[j] = gl < HALF ? g[j] * c[j] + partner * sn[j] : g[j] * c[j] - partner * sn[j];
      if (!qk) dn[j] = g[j];
    }
    float o[8];
    if (qk_norm) {
      const float r = qk ? rstd[it.t * (Hq + Hkv) + it.hh] : 0.f;
      float x[8];
      load8(kqv + it.t * C + it.col + gl * 8, x);
      const float* wv = it.kind == 0 ? wq : wk;
      float dot = 0.f, dxr[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        dxr[j] = dn[j] * wv[j];
        dot += dxr[j] * x[j];
      }
      dot = group_sum<LPH>(dot);
      const float c3 = dot * r * r * r / D;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j] = qk ? r * dxr[j] - x[j] * c3 : dn[j];
        const float contrib = valid ? dn[j] * rb(x[j] * r) : 0.f;
        if (it.kind == 0) accq[j] += contrib;
        else if (it.kind == 1) acck[j] += contrib;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = dn[j];
    }
    if (valid) store8(dkqv + it.t * C + it.col + gl * 8, o);
  }
  if (qk_norm) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      atomicAdd(&s_dqw[gl * 8 + j], accq[j]);
      atomicAdd(&s_dkw[gl * 8 + j], acck[j]);
    }
  }
  __syncthreads();
  if (qk_norm) {
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      atomicAdd(&dqw[i], s_dqw[i]);
      atomicAdd(&dkw[i], s_dkw[i]);
    }
  }
}

// ----------------------------------------------------------------- embedding
__global__ void embedding_fwd_k(const int64_t* __restrict__ ids, const bf16* __restrict__ table,
                                bf16* __restrict__ out, int64_t T, int H, int64_t V) {
  const int nv = H >> 3;
  const int64_t total = T * nv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nv;
    const int c = static_cast<int>(i % nv);
    int64_t id = ids[t];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);
    reinterpret_cast<uint4*>(out + t * H)[c] = reinterpret_cast<const uint4*>(table + id * H)[c];
  }
}

__global__ void embedding_bwd_k(const int64_t* __restrict__ ids, const bf16* __restrict__ dy,
                                float* __restrict__ dtable, int64_t T, int H, int64_t V) {
  const int nv = H >> 3;
  const int64_t total = T * nv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nv;
    const int c = static_cast<int>(i % nv);
    int64_t id = ids[t];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);
    float v[8];
    load8(dy + t * H + c * 8, v);
    float* dst = dtable + id * H + c * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(dst + j, v[j]);
  }
}

// ----------------------------------------------------------------- cross-entropy
__global__ void ce_loss_grad_k(bf16* __restrict__ logits, const float2* __restrict__ stats,
                               int ntiles, const int64_t* __restrict__ targets,
                               float* __restrict__ loss, const float* __restrict__ scale_p,
                               int64_t T, int V, int64_t ignore_index) {
  const int64_t row = blockIdx.x;
  if (row >= T) return;
  const int tid = threadIdx.x;
  const float2* st = stats + row * ntiles;
  // every thread reduces the (small) partial list redundantly -- no sync needed
  float m = -INFINITY;
  for (int i = 0; i < ntiles; ++i) m = fmaxf(m, st[i].x);
  float se = 0.f;
  for (int i = 0; i < ntiles; ++i) se += st[i].y * __expf(st[i].x - m);
  const float lse = m + __logf(se);
  const int64_t tgt = targets[row];
  const bool valid = tgt != ignore_index && tgt >= 0 && tgt < V;
  bf16* lr = logits + row * (int64_t)V;
  if (tid == 0) {
    loss[row] = valid ? lse - __bfloat162float(lr[tgt]) : 0.f;
  }
  const float scale = valid ? *scale_p : 0.f;
  const int nv = V >> 3;
  for (int i = tid; i < nv; i += blockDim.x) {
    float v[8];
    load8(lr + i * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p = __expf(v[j] - lse);
      if (i * 8 + j == tgt) p -= 1.f;
      v[j] = p * scale;
    }
    store8(lr + i * 8, v);
  }
}

// ----------------------------------------------------------------- routes
__global__ void route_scales_k(const int64_t* __restrict__ ids, const int64_t* __restrict__ table,
                               const float* __restrict__ rw, float* __restrict__ out, int64_t T,
                               int top_k, int64_t V, int E, float routed_scale) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t id = ids[t];
    id = id < 0 ? 0 : (id >= V ? V - 1 : id);
    float acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0.f;
    for (int j = 0; j < top_k; ++j) {
      const int64_t e = table[(int64_t)j * V + id];
#pragma unroll
      for (int q = 0; q < 16; ++q)
        if (q == e) acc[q] += rw[j];
    }
    for (int e = 0; e < E; ++e) out[t * E + e] = acc[e] * routed_scale;
  }
}

// ----------------------------------------------------------------- AdamW
__global__ void adamw_flat_k(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                             const bf16* __restrict__ g, bf16* __restrict__ p_out, int64_t n,
                             float lr, float b1, float b2, float eps, float wd, float bc1,
                             float bc2_sqrt, const float* __restrict__ clip) {
  const float cs = clip != nullptr ? *clip : 1.f;
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = __bfloat162float(g[i]) * cs;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = p[i] * decay;
    pi -= step * mi / (sqrtf(vi) / bc2_sqrt + eps);
    p[i] = pi;
    if (p_out != nullptr) p_out[i] = __float2bfloat16(pi);
  }
}

__global__ void sumsq_bf16_k(const bf16* __restrict__ g, int64_t n, float* __restrict__ out) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = __bfloat162float(g[i]);
    acc += x * x;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(out, v);
  }
}

__global__ void clip_coef_k(const float* sumsq, float max_norm, float* clip, float* norm) {
  const float nrm = sqrtf(*sumsq);
  if (norm != nullptr) *norm = nrm;
  if (clip != nullptr) *clip = max_norm > 0.f ? fminf(1.f, max_norm / (nrm + 1e-6f)) : 1.f;
}

}  // namespace

void rmsnorm_fwd(const bf16* x, const bf16* w, bf16* y, float* rstd, int64_t T, int H, float eps,
                 cudaStream_t s) {
  rmsnorm_fwd_k<<<grid_for(T, 8), 256, 0, s>>>(x, w, y, rstd, T, H, eps);
}

void rmsnorm_bwd(const bf16* dy, const bf16* x, const bf16* w, const float* rstd,
                 const bf16* dres, bf16* dx, float* dw, int64_t T, int H, cudaStream_t s) {
  const int nv = H / 8;
  const int grid = grid_for(T, 8, 148 * 3);
  const size_t sm = 2 * H * sizeof(float);
  if (nv <= 32)
    rmsnorm_bwd_reg_k<1><<<grid, 256, sm, s>>>(dy, x, w, rstd, dres, dx, dw, T, H);
  else if (nv <= 64)
    rmsnorm_bwd_reg_k<2><<<grid, 256, sm, s>>>(dy, x, w, rstd, dres, dx, dw, T, H);
  else if (nv <= 128)
    rmsnorm_bwd_reg_k<4><<<grid, 256, sm, s>>>(dy, x, w, rstd, dres, dx, dw, T, H);
  else
    rmsnorm_bwd_k<<<grid_for(T, 8, 148 * 8), 256, H * sizeof(float), s>>>(dy, x, w, rstd, dres,
                                                                         dx, dw, T, H);
}

void qk_norm_rope_fwd(const bf16* kqv, const bf16* qw, const bf16* kw, const float* cos_t,
                      const float* sin_t, const int32_t* pos, bf16* q, bf16* k, bf16* v,
                      float* rstd, int B, int S, int Hq, int Hkv, int D, float eps, bool qk_norm,
                      bool q_tm, cudaStream_t s) {
  const int64_t items = (int64_t)B * S * (Hq + 2 * Hkv);
  const int grid = grid_for(items, 8 * (256 / D), 148 * 16);
  if (D == 64)
    qk_norm_rope_fwd_k<64><<<grid, 256, 0, s>>>(kqv, qw, kw, cos_t, sin_t, pos, q, k, v, rstd, B, S,
                                               Hq, Hkv, eps, qk_norm, q_tm);
  else
    qk_norm_rope_fwd_k<128><<<grid, 256, 0, s>>>(kqv, qw, kw, cos_t, sin_t, pos, q, k, v, rstd, B, S,
                                               Hq, Hkv, eps, qk_norm, q_tm);
}

void qk_norm_rope_bwd(const bf16* dq, const bf16* dk, const bf16* dv, const bf16* kqv,
                      const bf16* qw, const bf16* kw, const float* cos_t, const float* sin_t,
                      const int32_t* pos, const float* rstd, bf16* dkqv, float* dqw, float* dkw,
                      int B, int S, int Hq, int Hkv, int D, bool qk_norm, bool q_tm,
                      cudaStream_t s) {
  const int64_t items = (int64_t)B * S * (Hq + 2 * Hkv);
  const int grid = grid_for(items, 8 * (256 / D), 148 * 3);
  if (D == 64)
    qk_norm_rope_bwd_k<64><<<grid, 256, 0, s>>>(dq, dk, dv, kqv, qw, kw, cos_t, sin_t, pos, rstd,
                                               dkqv, dqw, dkw, B, S, Hq, Hkv, qk_norm, q_tm);
  else
    qk_norm_rope_bwd_k<128><<<grid, 256, 0, s>>>(dq, dk, dv, kqv, qw, kw, cos_t, sin_t, pos, rstd,
                                               dkqv, dqw, dkw, B, S, Hq, Hkv, qk_norm, q_tm);
}

void embedding_fwd(const int64_t* ids, const bf16* table, bf16* out, int64_t T, int H, int64_t V,
                   cudaStream_t s) {
  embedding_fwd_k<<<grid_for(T * (H / 8), 256), 256, 0, s>>>(ids, table, out, T, H, V);
}

void embedding_bwd(const int64_t* ids, const bf16* dy, float* dtable, int64_t T, int H, int64_t V,
                   cudaStream_t s) {
  embedding_bwd_k<<<grid_for(T * (H / 8), 256), 256, 0, s>>>(ids, dy, dtable, T, H, V);
}

void ce_loss_grad(bf16* logits, const float* stats, int ntiles, const int64_t* targets,
                  float* loss, const float* scale, int64_t T, int V, int64_t ignore_index,
                  cudaStream_t s) {
  ce_loss_grad_k<<<static_cast<unsigned>(T), 256, 0, s>>>(
      logits, reinterpret_cast<const float2*>(stats), ntiles, targets, loss, scale, T, V,
      ignore_index);
}

void route_scales(const int64_t* ids, const int64_t* table, const float* route_w, float* out,
                  int64_t T, int top_k, int64_t V, int E, float routed_scale, cudaStream_t s) {
  route_scales_k<<<grid_for(T, 256), 256, 0, s>>>(ids, table, route_w, out, T, top_k, V, E,
                                                  routed_scale);
}

void adamw_flat(float* p, float* m, float* v, const bf16* g, bf16* p_out, int64_t n, float lr,
                float beta1, float beta2, float eps, float wd, float bc1, float bc2,
                const float* clip, cudaStream_t s) {
  adamw_flat_k<<<grid_for(n, 256, 148 * 8), 256, 0, s>>>(p, m, v, g, p_out, n, lr, beta1, beta2,
                                                         eps, wd, bc1, sqrtf(bc2), clip);
}

void sumsq_bf16(const bf16* g, int64_t n, float* out, cudaStream_t s) {
  sumsq_bf16_k<<<grid_for(n, 1024, 148 * 4), 1024, 0, s>>>(g, n, out);
}

void clip_coef(const float* sumsq, float max_norm, float* clip, float* norm, cudaStream_t s) {
  clip_coef_k<<<1, 1, 0, s>>>(sumsq, max_norm, clip, norm);
}

}  // namespace cfb
