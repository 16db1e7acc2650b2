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
#include <map>
#include <mutex>
#include <set>
#include <utility>

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
__device__ __forceinline__ void unpack8(const uint4& u, float* v) {
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z),
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

// Wide rows, few of them (decoding: 64 rows of 4096): one 256-thread CTA per
// row, the row held in registers (NC chunks of 8 per thread), block reduction.
template <int NC>
__global__ void __launch_bounds__(256) rmsnorm_fwd_row_k(const bf16* __restrict__ x,
                                                          const bf16* __restrict__ w,
                                                          bf16* __restrict__ y,
                                                          float* __restrict__ rstd, int H,
                                                          float eps) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * H;
  const int nv = H >> 3;
  float v[NC][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int i = threadIdx.x + c * 256;
    if (i < nv) {
      load8(xr + i * 8, v[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[c][j] * v[c][j];
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += red[k];
  const float r = rsqrtf(tot / H + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int i = threadIdx.x + c * 256;
    if (i < nv) {
      float wv[8];
      load8(w + i * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[c][j] = rb(v[c][j] * r) * wv[j];
      store8(y + row * H + i * 8, v[c]);
    }
  }
  if (threadIdx.x == 0) rstd[row] = r;
}

// out[m, n] = bf16(alpha * acc[n, m] (+ resid[m, n])): the transposed fp32
// result of a swapped-operand split-K GEMM, one 32 x 32 tile per block.
__global__ void __launch_bounds__(256) skinny_finish_k(const float* __restrict__ acc, int ldacc,
                                                        const bf16* __restrict__ resid,
                                                        bf16* __restrict__ out, int M, int N,
                                                        float alpha) {
  __shared__ float tile[32][33];
  const int n0 = blockIdx.x * 32, m0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int k = ty; k < 32; k += 8) {
    const int n = n0 + k, m = m0 + tx;
    tile[k][tx] = (n < N && m < M) ? acc[static_cast<int64_t>(n) * ldacc + m] : 0.f;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int m = m0 + k, n = n0 + tx;
    if (m < M && n < N) {
      const int64_t o = static_cast<int64_t>(m) * N + n;
      float v = alpha * tile[tx][k];
      if (resid != nullptr) v += __bfloat162float(resid[o]);
      out[o] = __float2bfloat16(v);
    }
  }
}

// act[t, c] = silu(g) * u * scale(t, c) from the transposed fp32 result of a
// swapped-operand split-K gate|up GEMM: acc[r, t] over the packed rows, gate
// column c at row (c / 128) * 256 + c % 128 and its up column 128 rows later.
// scale = shared_scale for c < shared_width, else row_scale[t, expert(c)].
// One 32 (c) x 32 (t) tile per block, transposed through shared memory.
__global__ void __launch_bounds__(256) skinny_swiglu_k(
    const float* __restrict__ acc, int ldacc, const float* __restrict__ row_scale,
    bf16* __restrict__ act, int T, int A, int shared_width, int expert_width, int n_experts,
    float shared_scale) {
  __shared__ float tg[32][33], tu[32][33];
  const int c0 = blockIdx.x * 32, t0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int k = ty; k < 32; k += 8) {
    const int c = c0 + k, t = t0 + tx;
    float g = 0.f, u = 0.f;
    if (c < A && t < T) {
      const int64_t rg = static_cast<int64_t>(c / 128) * 256 + c % 128;
      g = acc[rg * ldacc + t];
      u = acc[(rg + 128) * ldacc + t];
    }
    tg[k][tx] = g;
    tu[k][tx] = u;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + k, c = c0 + tx;
    if (t < T && c < A) {
      const float g = rb(tg[tx][k]), u = rb(tu[tx][k]);
      float sc = shared_scale;
      if (c >= shared_width)
        sc = row_scale[static_cast<int64_t>(t) * n_experts + (c - shared_width) / expert_width];
      act[static_cast<int64_t>(t) * A + c] = __float2bfloat16(g / (1.f + __expf(-g)) * u * sc);
    }
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
// Head index hh: [0,Hq) q heads, [Hq, Hq+Hkv) k heads, [Hq+Hkv, Hq+2Hkv) v
// heads; the fused projection output kqv stores columns in k | q | v order.
template <int LPH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Norm-weight gradients without a zero-fill or a cast launch: every block adds
// its partial into `acc` (fp32; zero on entry), the last block to arrive on
// `ticket` writes acc to the bf16 outputs (out0 for elements < n0, out1 for
// the rest) and re-zeroes acc and the ticket, so the slot is ready for the
// next launch that uses it.
__device__ void small_grad_finish(float* acc, int* ticket, int n, bf16* out0, int n0,
                                  bf16* out1) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const bf16 v = __float2bfloat16(__ldcg(acc + i));
    if (i < n0) out0[i] = v;
    else out1[i - n0] = v;
    acc[i] = 0.f;
  }
  if (threadIdx.x == 0) *ticket = 0;
}


// One warp per token.  Each warp owns a ring of NS token slots in shared
// memory and keeps NS-1 tokens of loads in flight with cp.async (16-byte
// pieces, no spin-wait: cp.async.wait_group retires them), so HBM latency is
// hidden without holding rows in registers.  Compute then reads shared memory
// only.  Lane layout: LPH = D/8 lanes per head, lane gl holding elements
// [4gl, 4gl+4) and their rotate-half partners [D/2+4gl, D/2+4gl+4), so RoPE is
// lane-local; a warp covers GPW = 32/LPH heads per pass (q heads, then k heads,
// in one uniform loop).  v heads are a plain copy.  Destination offsets are
// formed once per token.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void lds4(const bf16* p, float* v) {  // 4 bf16 (8 bytes)
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void st4(bf16* p, const float* v) {
  uint2 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void lds4f(const float* p, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
// bf16 rounding of two floats with one conversion
__device__ __forceinline__ void rb2(float& a, float& b) {
  const float2 f = unpack_bf16x2(pack_bf16x2(a, b));
  a = f.x;
  b = f.y;
}

// Per-token destination bases: q is head-major [B, Hq, S, D] or token-major
// [B, S, Hq, D] (q_tm); k/v are head-major [B, Hkv, S, D].
struct TokenBases {
  int64_t q, kv;     // element offsets of head 0
  int64_t q_stride;  // elements between consecutive q heads
};
__device__ __forceinline__ TokenBases token_bases(int b, int s, int S, int Hq, int Hkv, int D,
                                                  bool q_tm) {
  TokenBases tb;
  tb.q = q_tm ? ((int64_t)b * S + s) * Hq * D : ((int64_t)b * Hq * S + s) * D;
  tb.q_stride = q_tm ? D : (int64_t)S * D;
  tb.kv = ((int64_t)b * Hkv * S + s) * D;
  return tb;
}

// Forward slot: the token's whole fused k|q|v row (C = (Hq + 2 Hkv) D bf16),
// then its cos and sin table rows (D/2 floats each).
template <int D, int NS>
__global__ void __launch_bounds__(128) qk_norm_rope_fwd_k(
    const bf16* __restrict__ kqv, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t,
    const int32_t* __restrict__ pos, bf16* __restrict__ q, bf16* __restrict__ k,
    bf16* __restrict__ v, float* __restrict__ rstd, int B, int S, int Hq, int Hkv, float eps,
    bool qk_norm, bool q_tm) {
  constexpr int LPH = D / 8, GPW = 32 / LPH, H2 = D / 2;
  extern __shared__ __align__(16) unsigned char qk_smem[];
  __shared__ __align__(16) float s_w[2][D];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    s_w[0][i] = __bfloat162float(qw[i]);
    s_w[1][i] = __bfloat162float(kw[i]);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int grp = lane / LPH, gl = lane % LPH;
  const int Htot = Hq + 2 * Hkv, Hqk = Hq + Hkv;
  const int C = Htot * D;
  const int T = B * S;
  const int warp = threadIdx.x >> 5;
  const int wpb = blockDim.x >> 5;
  const int wid = blockIdx.x * wpb + warp;
  const int nw = gridDim.x * wpb;
  const int slot = C * 2 + D * 4;  // bytes
  unsigned char* ring = qk_smem + (size_t)warp * NS * slot;
  auto issue = [&](int i) {  // prefetch this warp's i-th token into slot i % NS
    const int t = wid + i * nw;
    if (t < T) {
      const bf16* src = kqv + (int64_t)t * C;
      unsigned char* dst = ring + (i % NS) * slot;
      for (int c = lane; c < C / 8; c += 32) cp_async16(dst + c * 16, src + c * 8);
      const int p = pos != nullptr ? pos[t] : t % S;
      if (lane < D / 4) {  // D/2 floats of cos then of sin: D/8 16-byte pieces each
        const float* tab = lane < D / 8 ? cos_t : sin_t;
        cp_async16(dst + C * 2 + lane * 16, tab + (int64_t)p * H2 + (lane % (D / 8)) * 4);
      }
    }
    cp_async_commit();
  };
  // this lane's norm weights (q, k) at its 8 element positions
  float wq[8], wk[8];
  lds4f(&s_w[0][4 * gl], wq);
  lds4f(&s_w[0][H2 + 4 * gl], wq + 4);
  lds4f(&s_w[1][4 * gl], wk);
  lds4f(&s_w[1][H2 + 4 * gl], wk + 4);
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) issue(i);
  for (int i = 0; wid + i * nw < T; ++i) {
    issue(i + NS - 1);
    cp_async_wait<NS - 1>();
    __syncwarp();
    const int t = wid + i * nw;
    const bf16* row = reinterpret_cast<const bf16*>(ring + (i % NS) * slot);
    const float* cs = reinterpret_cast<const float*>(row + C);
    const int b = t / S, s = t - b * S;
    const TokenBases tb = token_bases(b, s, S, Hq, Hkv, D, q_tm);
    float c[4], sn[4];
    lds4f(cs + 4 * gl, c);
    lds4f(cs + H2 + 4 * gl, sn);
    for (int h0 = 0; h0 < Hqk; h0 += GPW) {  // uniform trip count: shuffles stay convergent
      const int hh = min(h0 + grp, Hqk - 1);
      const bool valid = h0 + grp < Hqk;
      const bool isq = hh < Hq;
      const int col = isq ? (Hkv + hh) * D : (hh - Hq) * D;
      float x[8];
      lds4(row + col + 4 * gl, x);
      lds4(row + col + H2 + 4 * gl, x + 4);
      if (qk_norm) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
        ss = group_sum<LPH>(ss);
        const float r = rsqrtf(ss * (1.0f / D) + eps);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          float a = x[j] * r, bb = x[j + 1] * r;
          rb2(a, bb);
          a *= isq ? wq[j] : wk[j];
          bb *= isq ? wq[j + 1] : wk[j + 1];
          rb2(a, bb);
          x[j] = a;
          x[j + 1] = bb;
        }
        if (gl == 0 && valid) rstd[(int64_t)t * Hqk + hh] = r;
      }
      float lo[4], hi[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        lo[j] = x[j] * c[j] - x[j + 4] * sn[j];
        hi[j] = x[j + 4] * c[j] + x[j] * sn[j];
      }
      if (valid) {
        bf16* dst = isq ? q + tb.q + hh * tb.q_stride : k + tb.kv + (int64_t)(hh - Hq) * S * D;
        st4(dst + 4 * gl, lo);
        st4(dst + H2 + 4 * gl, hi);
      }
    }
    // v heads: copy
    const bf16* vrow = row + Hqk * D;
    for (int c8 = lane; c8 < Hkv * D / 8; c8 += 32) {
      const int h = c8 / (D / 8), e = (c8 % (D / 8)) * 8;
      *reinterpret_cast<uint4*>(v + tb.kv + (int64_t)h * S * D + e) =
          *reinterpret_cast<const uint4*>(vrow + h * D + e);
    }
    __syncwarp();  // the slot is refilled by the next iteration's prefetch
  }
  cp_async_wait<0>();
}

// Backward slot: the gradients of all Htot heads in q, k, v head order (head
// hh at hh * D), the k|q part of the forward input row (only with qk_norm),
// the cos and sin rows, and the token's saved 1/rms values (Hq + Hkv floats,
// padded to 16 bytes).
template <int D, int NS>
__global__ void __launch_bounds__(128) qk_norm_rope_bwd_k(
    const bf16* __restrict__ dq, const bf16* __restrict__ dk, const bf16* __restrict__ dv,
    const bf16* __restrict__ kqv, const bf16* __restrict__ qw, const bf16* __restrict__ kw,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t,
    const int32_t* __restrict__ pos, const float* __restrict__ rstd, bf16* __restrict__ dkqv,
    float* __restrict__ dqw, float* __restrict__ dkw, int B, int S, int Hq, int Hkv,
    bool qk_norm, bool q_tm, bf16* dqw_out, bf16* dkw_out, int* ticket) {
  constexpr int LPH = D / 8, GPW = 32 / LPH, H2 = D / 2;
  extern __shared__ __align__(16) unsigned char qk_smem[];
  __shared__ float s_dqw[D], s_dkw[D];
  __shared__ __align__(16) float s_w[2][D];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    s_dqw[i] = 0.f;
    s_dkw[i] = 0.f;
    s_w[0][i] = __bfloat162float(qw[i]);
    s_w[1][i] = __bfloat162float(kw[i]);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int grp = lane / LPH, gl = lane % LPH;
  const int Htot = Hq + 2 * Hkv, Hqk = Hq + Hkv;
  const int C = Htot * D;
  const int CX = qk_norm ? Hqk * D : 0;  // k|q columns of the input row
  const int slot = (C + CX) * 2 + D * 4 + ((Hqk * 4 + 15) & ~15);  // bytes
  const int T = B * S;
  const int warp = threadIdx.x >> 5;
  const int wpb = blockDim.x >> 5;
  const int wid = blockIdx.x * wpb + warp;
  const int nw = gridDim.x * wpb;
  unsigned char* ring = qk_smem + (size_t)warp * NS * slot;
  auto issue = [&](int i) {
    const int t = wid + i * nw;
    if (t < T) {
      const int b = t / S, s = t - b * S;
      const TokenBases tb = token_bases(b, s, S, Hq, Hkv, D, q_tm);
      bf16* dst = reinterpret_cast<bf16*>(ring + (i % NS) * slot);
      for (int c8 = lane; c8 < Htot * LPH; c8 += 32) {
        const int hh = c8 / LPH, e = (c8 % LPH) * 8;
        const bf16* src = hh < Hq ? dq + tb.q + hh * tb.q_stride
                                  : (hh < Hqk ? dk + tb.kv + (int64_t)(hh - Hq) * S * D
                                              : dv + tb.kv + (int64_t)(hh - Hqk) * S * D);
        cp_async16(dst + hh * D + e, src + e);
      }
      const bf16* xr = kqv + (int64_t)t * C;
      for (int c8 = lane; c8 < CX / 8; c8 += 32) cp_async16(dst + C + c8 * 8, xr + c8 * 8);
      float* fdst = reinterpret_cast<float*>(dst + C + CX);
      const int p = pos != nullptr ? pos[t] : s;
      if (lane < D / 4) {
        const float* tab = lane < D / 8 ? cos_t : sin_t;
        cp_async16(fdst + lane * 4, tab + (int64_t)p * H2 + (lane % (D / 8)) * 4);
      }
      if (qk_norm)
        for (int c = lane; c < Hqk; c += 32) cp_async4(fdst + D + c, rstd + (int64_t)t * Hqk + c);
    }
    cp_async_commit();
  };
  float wq[8], wk[8], accq[8], acck[8];
  lds4f(&s_w[0][4 * gl], wq);
  lds4f(&s_w[0][H2 + 4 * gl], wq + 4);
  lds4f(&s_w[1][4 * gl], wk);
  lds4f(&s_w[1][H2 + 4 * gl], wk + 4);
#pragma unroll
  for (int j = 0; j < 8; ++j) accq[j] = acck[j] = 0.f;
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) issue(i);
  for (int i = 0; wid + i * nw < T; ++i) {
    issue(i + NS - 1);
    cp_async_wait<NS - 1>();
    __syncwarp();
    const int t = wid + i * nw;
    const bf16* sl = reinterpret_cast<const bf16*>(ring + (i % NS) * slot);
    const float* fs = reinterpret_cast<const float*>(sl + C + CX);
    bf16* drow = dkqv + (int64_t)t * C;
    float c[4], sn[4];
    lds4f(fs + 4 * gl, c);
    lds4f(fs + H2 + 4 * gl, sn);
    for (int h0 = 0; h0 < Hqk; h0 += GPW) {  // uniform trip count: shuffles stay convergent
      const int hh = min(h0 + grp, Hqk - 1);
      const bool valid = h0 + grp < Hqk;
      const bool isq = hh < Hq;
      const int col = isq ? (Hkv + hh) * D : (hh - Hq) * D;
      float g[8];
      lds4(sl + hh * D + 4 * gl, g);
      lds4(sl + hh * D + H2 + 4 * gl, g + 4);
      // inverse rotation
      float dn[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dn[j] = g[j] * c[j] + g[j + 4] * sn[j];
        dn[j + 4] = g[j + 4] * c[j] - g[j] * sn[j];
      }
      float o[8];
      if (qk_norm) {
        float x[8];
        lds4(sl + C + col + 4 * gl, x);
        lds4(sl + C + col + H2 + 4 * gl, x + 4);
        const float rr = fs[D + hh];
        float dot = 0.f, dxr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          dxr[j] = dn[j] * (isq ? wq[j] : wk[j]);
          dot += dxr[j] * x[j];
        }
        dot = group_sum<LPH>(dot);
        const float c3 = dot * rr * rr * rr * (1.0f / D);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          o[j] = rr * dxr[j] - x[j] * c3;
          o[j + 1] = rr * dxr[j + 1] - x[j + 1] * c3;
          float a = x[j] * rr, bb = x[j + 1] * rr;
          rb2(a, bb);
          const float ca = valid ? dn[j] * a : 0.f, cb = valid ? dn[j + 1] * bb : 0.f;
          accq[j] += isq ? ca : 0.f;
          accq[j + 1] += isq ? cb : 0.f;
          acck[j] += isq ? 0.f : ca;
          acck[j + 1] += isq ? 0.f : cb;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = dn[j];
      }
      if (valid) {
        st4(drow + col + 4 * gl, o);
        st4(drow + col + H2 + 4 * gl, o + 4);
      }
    }
    // v heads: the gradient passes through unchanged
    for (int c8 = lane; c8 < Hkv * D / 8; c8 += 32)
      *reinterpret_cast<uint4*>(drow + Hqk * D + c8 * 8) =
          *reinterpret_cast<const uint4*>(sl + Hqk * D + c8 * 8);
    __syncwarp();
  }
  cp_async_wait<0>();
  if (qk_norm) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = j < 4 ? 4 * gl + j : H2 + 4 * gl + (j - 4);
      atomicAdd(&s_dqw[e], accq[j]);
      atomicAdd(&s_dkw[e], acck[j]);
    }
  }
  __syncthreads();
  if (qk_norm) {
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      atomicAdd(&dqw[i], s_dqw[i]);
      atomicAdd(&dkw[i], s_dkw[i]);
    }
    // dkw == dqw + D when the outputs are bf16 (one accumulator slot)
    if (dqw_out != nullptr) small_grad_finish(dqw, ticket, 2 * D, dqw_out, D, dkw_out);
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

// Embedding backward over token ids sorted ascending (`order` maps sorted
// position -> token row): a warp takes 32 consecutive sorted positions,
// accumulates runs of equal ids in registers and adds each run into dtable
// with one vector reduction per 4 floats.  Frequent ids (Zipf-distributed
// text) then cost one atomic row-add per warp instead of one per token.
template <int NV>
__global__ void __launch_bounds__(256) embedding_bwd_sorted_k(
    const int64_t* __restrict__ sorted_ids, const int64_t* __restrict__ order,
    const bf16* __restrict__ dy, float* __restrict__ dtable, int64_t T, int H, int64_t V) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t p0 = warp * 32;
  if (p0 >= T) return;
  const int nv = H / 8;
  const int64_t pl = p0 + lane;
  // clamped like the forward; clamped ids still form contiguous runs
  int64_t my_id = pl < T ? sorted_ids[pl] : 0;
  my_id = my_id < 0 ? 0 : (my_id >= V ? V - 1 : my_id);
  const int64_t my_row = pl < T ? order[pl] : 0;
  const int n = T - p0 < 32 ? static_cast<int>(T - p0) : 32;
  float acc[NV][8];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
  int64_t cur = __shfl_sync(0xffffffffu, my_id, 0);
  auto flush = [&](int64_t id) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < nv) {
        float* dst = dtable + id * H + i * 8;
        red_add_v4(dst, acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
        red_add_v4(dst + 4, acc[k][4], acc[k][5], acc[k][6], acc[k][7]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
    }
  };
  for (int q = 0; q < n; ++q) {
    const int64_t id = __shfl_sync(0xffffffffu, my_id, q);
    const int64_t row = __shfl_sync(0xffffffffu, my_row, q);
    if (id != cur) {  // warp-uniform
      flush(cur);
      cur = id;
    }
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < nv) {
        float v[8];
        load8(dy + row * H + i * 8, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[k][j] += v[j];
      }
    }
  }
  flush(cur);
}

// ----------------------------------------------------------------- cross-entropy
// One 256-thread block per row.  The row's per-128-column partials (max,
// sum of exp) are combined cooperatively (one partial per thread, then block
// max / sum), and the gradient pass keeps four 16-byte vectors per thread in
// flight.
__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) v = is_max ? fmaxf(v, red[i]) : v + red[i];
  __syncthreads();  // red is reused by the next reduction
  return v;
}

__global__ void __launch_bounds__(256) ce_loss_grad_k(
    bf16* __restrict__ logits, const float2* __restrict__ stats, int ntiles,
    const int64_t* __restrict__ targets, float* __restrict__ loss,
    const float* __restrict__ scale_p, int64_t T, int V, int64_t ignore_index) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  if (row >= T) return;
  const int tid = threadIdx.x;
  const float2* st = stats + row * ntiles;
  float m = -INFINITY;
  for (int i = tid; i < ntiles; i += blockDim.x) m = fmaxf(m, st[i].x);
  m = block_reduce(m, true, red);
  float se = 0.f;
  for (int i = tid; i < ntiles; i += blockDim.x) se += st[i].y * __expf(st[i].x - m);
  se = block_reduce(se, false, red);
  const float lse = m + __logf(se);
  const int64_t tgt = targets[row];
  const bool valid = tgt != ignore_index && tgt >= 0 && tgt < V;
  bf16* lr = logits + row * (int64_t)V;
  if (tid == 0) loss[row] = valid ? lse - __bfloat162float(lr[tgt]) : 0.f;
  __syncthreads();  // the target logit is read before any thread overwrites it
  const float scale = valid ? *scale_p : 0.f;
  const int nv = V >> 3;
  constexpr int U = 4;
  for (int i0 = tid; i0 < nv; i0 += U * blockDim.x) {
    float v[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < nv) load8(lr + i * 8, v[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < nv) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float p = __expf(v[u][j] - lse);
          if (i * 8 + j == tgt) p -= 1.f;
          v[u][j] = p * scale;
        }
        store8(lr + i * 8, v[u]);
      }
    }
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
__device__ __forceinline__ float adamw_elem(float& p, float& m, float& v, float g, float b1,
                                            float b2, float eps, float decay, float step,
                                            float bc2_sqrt) {
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  p = p * decay - step * m / (sqrtf(v) / bc2_sqrt + eps);
  return p;
}

// 8 elements per thread per iteration with 16-byte accesses (the buffers are
// flat and 128-element aligned); a scalar loop takes any ragged tail.
__global__ void __launch_bounds__(256) adamw_flat_k(float* __restrict__ p, float* __restrict__ m,
                                                    float* __restrict__ v,
                                                    const bf16* __restrict__ g,
                                                    bf16* __restrict__ p_out, int64_t n, float lr,
                                                    float b1, float b2, float eps, float wd,
                                                    float bc1, float bc2_sqrt,
                                                    const float* __restrict__ clip,
                                                    const float* __restrict__ hyper, bool vec) {
  const float cs = clip != nullptr ? *clip : 1.f;
  if (hyper != nullptr) {
    lr = hyper[0];
    bc1 = hyper[1];
    bc2_sqrt = sqrtf(hyper[2]);
  }
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  const int64_t nv = vec ? n / 8 : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4* p4 = reinterpret_cast<float4*>(p) + 2 * i;
    float4* m4 = reinterpret_cast<float4*>(m) + 2 * i;
    float4* v4 = reinterpret_cast<float4*>(v) + 2 * i;
    float pv[8], mv[8], vv[8], gv[8];
    const float4 pa = p4[0], pb = p4[1], ma = m4[0], mb = m4[1], va = v4[0], vb = v4[1];
    load8(g + 8 * i, gv);
    pv[0] = pa.x; pv[1] = pa.y; pv[2] = pa.z; pv[3] = pa.w;
    pv[4] = pb.x; pv[5] = pb.y; pv[6] = pb.z; pv[7] = pb.w;
    mv[0] = ma.x; mv[1] = ma.y; mv[2] = ma.z; mv[3] = ma.w;
    mv[4] = mb.x; mv[5] = mb.y; mv[6] = mb.z; mv[7] = mb.w;
    vv[0] = va.x; vv[1] = va.y; vv[2] = va.z; vv[3] = va.w;
    vv[4] = vb.x; vv[5] = vb.y; vv[6] = vb.z; vv[7] = vb.w;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      adamw_elem(pv[j], mv[j], vv[j], gv[j] * cs, b1, b2, eps, decay, step, bc2_sqrt);
    p4[0] = make_float4(pv[0], pv[1], pv[2], pv[3]);
    p4[1] = make_float4(pv[4], pv[5], pv[6], pv[7]);
    m4[0] = make_float4(mv[0], mv[1], mv[2], mv[3]);
    m4[1] = make_float4(mv[4], mv[5], mv[6], mv[7]);
    v4[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    v4[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
    if (p_out != nullptr) store8(p_out + 8 * i, pv);
  }
  for (int64_t i = nv * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float pi = p[i], mi = m[i], vi = v[i];
    adamw_elem(pi, mi, vi, __bfloat162float(g[i]) * cs, b1, b2, eps, decay, step, bc2_sqrt);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (p_out != nullptr) p_out[i] = __float2bfloat16(pi);
  }
}

__global__ void sumsq_bf16_k(const bf16* __restrict__ g, int64_t n, float* __restrict__ out,
                             bool vec) {
  __shared__ float red[32];
  float acc = 0.f;
  const int64_t nv = vec ? n / 8 : 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv;
       i += (int64_t)gridDim.x * blockDim.x) {
    float x[8];
    load8(g + 8 * i, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += x[j] * x[j];
  }
  for (int64_t i = nv * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
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

// RMSNorm for H <= 1024 with the warp-owned cp.async ring of the QK kernels:
// a warp streams its rows through NS shared-memory slots (NS-1 rows of loads
// in flight) and computes from shared memory.  Lane l owns the 8-element
// vectors l, l+32, ... (NV of them) of a row; in backward its d(weight)
// partials stay in registers for the whole row loop.
template <int NV, int NS>
__global__ void __launch_bounds__(128) rmsnorm_fwd_ring_k(const bf16* __restrict__ x,
                                                         const bf16* __restrict__ w,
                                                         bf16* __restrict__ y,
                                                         float* __restrict__ rstd, int T, int H,
                                                         float eps) {
  extern __shared__ __align__(16) unsigned char rn_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int wid = blockIdx.x * wpb + warp, nw = gridDim.x * wpb;
  const int nv = H / 8;
  bf16* ring = reinterpret_cast<bf16*>(rn_smem) + (size_t)warp * NS * H;
  float wv[NV][8];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = lane + 32 * k;
    if (i < nv) load8(w + i * 8, wv[k]);
  }
  auto issue = [&](int it) {
    const int row = wid + it * nw;
    if (row < T) {
      const bf16* src = x + (int64_t)row * H;
      bf16* dst = ring + (it % NS) * H;
      for (int i = lane; i < nv; i += 32) cp_async16(dst + i * 8, src + i * 8);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int it = 0; it < NS - 1; ++it) issue(it);
  for (int it = 0; wid + it * nw < T; ++it) {
    issue(it + NS - 1);
    cp_async_wait<NS - 1>();
    __syncwarp();
    const int row = wid + it * nw;
    const bf16* xr = ring + (it % NS) * H;
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < nv) {
        load8(xr + i * 8, v[k]);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += v[k][j] * v[k][j];
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / H + eps);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < nv) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[k][j] = rb(v[k][j] * r) * wv[k][j];
        store8(y + (int64_t)row * H + i * 8, v[k]);
      }
    }
    if (lane == 0) rstd[row] = r;
    __syncwarp();
  }
  cp_async_wait<0>();
}

template <int NV, int NS>
__global__ void __launch_bounds__(128) rmsnorm_bwd_ring_k(
    const bf16* __restrict__ dy, const bf16* __restrict__ x, const bf16* __restrict__ w,
    const float* __restrict__ rstd, const bf16* __restrict__ dres, bf16* __restrict__ dx,
    float* __restrict__ dw, int T, int H, bf16* dw_out, int* ticket) {
  extern __shared__ __align__(16) unsigned char rn_smem[];
  float* sdw = reinterpret_cast<float*>(rn_smem);  // [H] block partials of d(weight)
  float* sw = sdw + H;                               // [H] weights
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int wid = blockIdx.x * wpb + warp, nw = gridDim.x * wpb;
  const int nv = H / 8;
  const int rows = dres != nullptr ? 3 : 2;
  const int slot = rows * H * 2 + 16;  // bytes: dy | x | dres rows, then rstd
  unsigned char* ring = rn_smem + 2 * H * sizeof(float) + (size_t)warp * NS * slot;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    sdw[i] = 0.f;
    sw[i] = __bfloat162float(w[i]);
  }
  __syncthreads();
  float acc[NV][8];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
  auto wload = [&](int i, float* wv) {
    const float4 a = *reinterpret_cast<const float4*>(sw + i * 8);
    const float4 b = *reinterpret_cast<const float4*>(sw + i * 8 + 4);
    wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
    wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
  };
  auto issue = [&](int it) {
    const int row = wid + it * nw;
    if (row < T) {
      bf16* dst = reinterpret_cast<bf16*>(ring + (it % NS) * slot);
      const int64_t o = (int64_t)row * H;
      for (int i = lane; i < nv; i += 32) {
        cp_async16(dst + i * 8, dy + o + i * 8);
        cp_async16(dst + H + i * 8, x + o + i * 8);
        if (dres != nullptr) cp_async16(dst + 2 * H + i * 8, dres + o + i * 8);
      }
      if (lane == 0) cp_async4(dst + rows * H, rstd + row);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int it = 0; it < NS - 1; ++it) issue(it);
  for (int it = 0; wid + it * nw < T; ++it) {
    issue(it + NS - 1);
    cp_async_wait<NS - 1>();
    __syncwarp();
    const int row = wid + it * nw;
    const bf16* sl = reinterpret_cast<const bf16*>(ring + (it % NS) * slot);
    const float r = *reinterpret_cast<const float*>(sl + rows * H);
    float dot = 0.f;
    // this lane's x / dy vectors stay in registers (packed bf16) for the second
    // pass instead of being read from shared memory again
    uint4 xq[NV], gq[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = lane + 32 * k;
      if (i < nv) {
        float xv[8], gv[8], wv[8];
        xq[k] = *reinterpret_cast<const uint4*>(sl + H + i * 8);
        gq[k] = *reinterpret_cast<const uint4*>(sl + i * 8);
        unpack8(xq[k], xv);
        unpack8(gq[k], gv);
        wload(i, wv);
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
        float xv[8], gv[8], wv[8], o[8];
        unpack8(xq[k], xv);
        unpack8(gq[k], gv);
        wload(i, wv);
        if (dres != nullptr) {
          load8(sl + 2 * H + i * 8, o);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += r * gv[j] * wv[j] - xv[j] * c;
        store8(dx + (int64_t)row * H + i * 8, o);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
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
  if (dw_out != nullptr) small_grad_finish(dw, ticket, H, dw_out, H, nullptr);
}

}  // namespace

// Grid of one resident wave for a ring kernel with `smem` bytes per 4-warp block.
template <typename K>
static int ring_grid(K kern, size_t smem, int64_t rows) {
  static std::mutex mu;
  static std::map<std::pair<const void*, size_t>, int> cache;
  const void* fn = reinterpret_cast<const void*>(kern);
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({fn, smem});
    if (it != cache.end()) {
      per_sm = it->second;
    } else {
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 128, smem) != cudaSuccess ||
          per_sm < 1)
        per_sm = 1;
      cache[{fn, smem}] = per_sm;
    }
  }
  return grid_for(rows, 4, 148 * per_sm);
}

constexpr int kRnStages = 4;

void rmsnorm_fwd(const bf16* x, const bf16* w, bf16* y, float* rstd, int64_t T, int H, float eps,
                 cudaStream_t s) {
  const int nv = H / 8;
  if (nv <= 128 && T < (int64_t(1) << 31)) {
    const size_t smem = (size_t)4 * kRnStages * H * sizeof(bf16);
    auto kern = nv <= 32 ? rmsnorm_fwd_ring_k<1, kRnStages>
                : nv <= 64 ? rmsnorm_fwd_ring_k<2, kRnStages> : rmsnorm_fwd_ring_k<4, kRnStages>;
    kern<<<ring_grid(kern, smem, T), 128, smem, s>>>(x, w, y, rstd, static_cast<int>(T), H, eps);
    return;
  }
  if (T <= 8192 && nv <= 4 * 256 && T < (int64_t(1) << 31)) {
    const int nc = (nv + 255) / 256;
    if (nc == 1) rmsnorm_fwd_row_k<1><<<T, 256, 0, s>>>(x, w, y, rstd, H, eps);
    else if (nc == 2) rmsnorm_fwd_row_k<2><<<T, 256, 0, s>>>(x, w, y, rstd, H, eps);
    else rmsnorm_fwd_row_k<4><<<T, 256, 0, s>>>(x, w, y, rstd, H, eps);
    return;
  }
  rmsnorm_fwd_k<<<grid_for(T, 8), 256, 0, s>>>(x, w, y, rstd, T, H, eps);
}

void skinny_swiglu(const float* acc, int ldacc, const float* row_scale, bf16* act, int T, int A,
                   int shared_width, int expert_width, int n_experts, float shared_scale,
                   cudaStream_t s) {
  skinny_swiglu_k<<<dim3((A + 31) / 32, (T + 31) / 32), 256, 0, s>>>(
      acc, ldacc, row_scale, act, T, A, shared_width, expert_width, n_experts, shared_scale);
}

void skinny_finish(const float* acc, int ldacc, const bf16* resid, bf16* out, int M, int N,
                   float alpha, cudaStream_t s) {
  skinny_finish_k<<<dim3((N + 31) / 32, (M + 31) / 32), 256, 0, s>>>(acc, ldacc, resid, out, M,
                                                                     N, alpha);
}

void rmsnorm_bwd(const bf16* dy, const bf16* x, const bf16* w, const float* rstd,
                 const bf16* dres, bf16* dx, float* dw, int64_t T, int H, bf16* dw_out,
                 int* ticket, cudaStream_t s) {
  const int nv = H / 8;
  if (nv <= 128 && T < (int64_t(1) << 31)) {
    const int rows = dres != nullptr ? 3 : 2;
    // two stages: the compute from shared memory needs the warps more than a
    // third row in flight (measured 52 vs 54 us at T=32768, H=896)
    constexpr int ns = 2;
    const size_t smem = 2 * H * sizeof(float) + (size_t)4 * ns * (rows * H * 2 + 16);
    auto kern = nv <= 32 ? rmsnorm_bwd_ring_k<1, ns>
                : nv <= 64 ? rmsnorm_bwd_ring_k<2, ns> : rmsnorm_bwd_ring_k<4, ns>;
    kern<<<ring_grid(kern, smem, T), 128, smem, s>>>(dy, x, w, rstd, dres, dx, dw,
                                                     static_cast<int>(T), H, dw_out, ticket);
    return;
  }
  if (dw_out != nullptr) return;  // bf16 outputs exist only on the ring path (checked by callers)
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

// Launch shape of the cp.async ring kernels: 4 warps x 4 stages, fewer when a
// token slot is large (many heads), so the ring fits in shared memory.
struct QkLaunch {
  int warps, stages, grid;
  size_t smem;
};

template <typename K4, typename K2>
QkLaunch qk_launch(K4 k4, K2 k2, int slot_bytes, int64_t tokens) {
  constexpr size_t kMaxSmem = 200 * 1024;
  QkLaunch L{4, 4, 1, 0};
  const size_t slot = (size_t)slot_bytes;
  while (L.warps * L.stages * slot > kMaxSmem && (L.stages > 2 || L.warps > 1)) {
    if (L.warps > 1) L.warps >>= 1;
    else L.stages = 2;
  }
  L.smem = L.warps * L.stages * slot;
  // The size attribute is raised once per kernel to the cap (it bounds, but
  // does not set, the launch's shared memory); occupancy is cached per shape.
  static std::mutex mu;
  static std::set<const void*> raised;
  static std::map<std::pair<const void*, size_t>, int> per_sm_cache;
  const void* fn = L.stages == 4 ? reinterpret_cast<const void*>(k4)
                                 : reinterpret_cast<const void*>(k2);
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (raised.insert(fn).second)
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    const std::pair<const void*, size_t> key{fn, L.smem * 8 + L.warps};
    auto it = per_sm_cache.find(key);
    if (it != per_sm_cache.end()) {
      per_sm = it->second;
    } else {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, L.warps * 32, L.smem) !=
              cudaSuccess ||
          per_sm < 1)
        per_sm = 1;
      per_sm_cache[key] = per_sm;
    }
  }
  L.grid = grid_for(tokens, L.warps, 148 * per_sm);  // one resident wave
  return L;
}

void qk_norm_rope_fwd(const bf16* kqv, const bf16* qw, const bf16* kw, const float* cos_t,
                      const float* sin_t, const int32_t* pos, bf16* q, bf16* k, bf16* v,
                      float* rstd, int B, int S, int Hq, int Hkv, int D, float eps, bool qk_norm,
                      bool q_tm, cudaStream_t s) {
  const int slot = (Hq + 2 * Hkv) * D * 2 + D * 4;  // bytes; matches the kernel
  const int64_t T = (int64_t)B * S;
#define CFB_QK_FWD(DD)                                                                          \
  {                                                                                             \
    const QkLaunch L = qk_launch(qk_norm_rope_fwd_k<DD, 4>, qk_norm_rope_fwd_k<DD, 2>, slot, T); \
    auto kern = L.stages == 4 ? qk_norm_rope_fwd_k<DD, 4> : qk_norm_rope_fwd_k<DD, 2>;          \
    kern<<<L.grid, L.warps * 32, L.smem, s>>>(kqv, qw, kw, cos_t, sin_t, pos, q, k, v, rstd, B,  \
                                              S, Hq, Hkv, eps, qk_norm, q_tm);                  \
  }
  if (D == 64) CFB_QK_FWD(64) else CFB_QK_FWD(128)
#undef CFB_QK_FWD
}

void qk_norm_rope_bwd(const bf16* dq, const bf16* dk, const bf16* dv, const bf16* kqv,
                      const bf16* qw, const bf16* kw, const float* cos_t, const float* sin_t,
                      const int32_t* pos, const float* rstd, bf16* dkqv, float* dqw, float* dkw,
                      int B, int S, int Hq, int Hkv, int D, bool qk_norm, bool q_tm,
                      bf16* dqw_out, bf16* dkw_out, int* ticket, cudaStream_t s) {
  const int nr = Hq + Hkv;  // bytes; matches the kernel
  const int slot = ((Hq + 2 * Hkv) * D + (qk_norm ? nr * D : 0)) * 2 + D * 4 + ((nr * 4 + 15) & ~15);
  const int64_t T = (int64_t)B * S;
#define CFB_QK_BWD(DD)                                                                          \
  {                                                                                             \
    const QkLaunch L = qk_launch(qk_norm_rope_bwd_k<DD, 4>, qk_norm_rope_bwd_k<DD, 2>, slot, T); \
    auto kern = L.stages == 4 ? qk_norm_rope_bwd_k<DD, 4> : qk_norm_rope_bwd_k<DD, 2>;          \
    kern<<<L.grid, L.warps * 32, L.smem, s>>>(dq, dk, dv, kqv, qw, kw, cos_t, sin_t, pos, rstd,  \
                                              dkqv, dqw, dkw, B, S, Hq, Hkv, qk_norm, q_tm,     \
                                              dqw_out, dkw_out, ticket);                        \
  }
  if (D == 64) CFB_QK_BWD(64) else CFB_QK_BWD(128)
#undef CFB_QK_BWD
}

void embedding_fwd(const int64_t* ids, const bf16* table, bf16* out, int64_t T, int H, int64_t V,
                   cudaStream_t s) {
  embedding_fwd_k<<<grid_for(T * (H / 8), 256), 256, 0, s>>>(ids, table, out, T, H, V);
}

void embedding_bwd(const int64_t* ids, const bf16* dy, float* dtable, int64_t T, int H, int64_t V,
                   cudaStream_t s) {
  embedding_bwd_k<<<grid_for(T * (H / 8), 256), 256, 0, s>>>(ids, dy, dtable, T, H, V);
}

void embedding_bwd_sorted(const int64_t* sorted_ids, const int64_t* order, const bf16* dy,
                          float* dtable, int64_t T, int H, int64_t V, cudaStream_t s) {
  const int nv = H / 8;
  const unsigned grid = static_cast<unsigned>((T + 255) / 256);  // 8 warps x 32 positions
  if (nv <= 32)
    embedding_bwd_sorted_k<1><<<grid, 256, 0, s>>>(sorted_ids, order, dy, dtable, T, H, V);
  else if (nv <= 64)
    embedding_bwd_sorted_k<2><<<grid, 256, 0, s>>>(sorted_ids, order, dy, dtable, T, H, V);
  else
    embedding_bwd_sorted_k<4><<<grid, 256, 0, s>>>(sorted_ids, order, dy, dtable, T, H, V);
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
                const float* clip, const float* hyper, cudaStream_t s) {
  auto al = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  const bool vec = al(p) && al(m) && al(v) && al(g) && (p_out == nullptr || al(p_out));
  adamw_flat_k<<<grid_for(vec ? n / 8 + 1 : n, 256, 148 * 8), 256, 0, s>>>(
      p, m, v, g, p_out, n, lr, beta1, beta2, eps, wd, bc1, sqrtf(bc2), clip, hyper, vec);
}

void sumsq_bf16(const bf16* g, int64_t n, float* out, cudaStream_t s) {
  const bool vec = reinterpret_cast<uintptr_t>(g) % 16 == 0;
  sumsq_bf16_k<<<grid_for(vec ? n / 8 + 1 : n, 1024, 148 * 4), 1024, 0, s>>>(g, n, out, vec);
}

void clip_coef(const float* sumsq, float max_norm, float* clip, float* norm, cudaStream_t s) {
  clip_coef_k<<<1, 1, 0, s>>>(sumsq, max_norm, clip, norm);
}

}  // namespace cfb
