// Host launchers of the memory-bound sm_100a kernels (elementwise.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cfb {

using bf16 = __nv_bfloat16;

// RMSNorm over the last dim H (H % 8 == 0).  y = bf16(bf16(x*rstd) * w).
// out[m, n] = bf16(alpha * acc[n, m] (+ resid[m, n])) for m < M, n < N (acc row stride ldacc).
void skinny_finish(const float* acc, int ldacc, const bf16* resid, bf16* out, int M, int N,
                   float alpha, cudaStream_t s);
// act[t, c] = silu(g) * u * scale(t, c) from acc [2A packed gate|up rows, >= T] (fp32,
// row stride ldacc): gate row of c = (c/128)*256 + c%128, up row 128 later.
void skinny_swiglu(const float* acc, int ldacc, const float* row_scale, bf16* act, int T, int A,
                   int shared_width, int expert_width, int n_experts, float shared_scale,
                   cudaStream_t s);
void rmsnorm_fwd(const bf16* x, const bf16* w, bf16* y, float* rstd, int64_t T, int H, float eps,
                 cudaStream_t s);
// dx = rmsnorm'(x)^T dy (+ dres);  dw (fp32, [H]) += sum_rows dy * x*rstd.
// With dw_out (H <= 1024): dw is a zeroed accumulator slot with a zeroed
// ticket; the last block writes bf16 dw_out and re-zeroes both.
void rmsnorm_bwd(const bf16* dy, const bf16* x, const bf16* w, const float* rstd,
                 const bf16* dres, bf16* dx, float* dw, int64_t T, int H, bf16* dw_out,
                 int* ticket, cudaStream_t s);

// kqv [T, (2*Hkv+Hq)*D] in k|q|v order -> per-head RMSNorm of q and k, RoPE
// (rotate-half, cos/sin tables [P, D/2]) and scatter to head-major k/v
// [B, H, S, D] and q (head-major, or token-major [B, S, Hq, D] with q_tm).  rstd [T, Hq+Hkv] (q heads first).
void qk_norm_rope_fwd(const bf16* kqv, const bf16* qw, const bf16* kw, const float* cos_t,
                      const float* sin_t, const int32_t* pos, bf16* q, bf16* k, bf16* v,
                      float* rstd, int B, int S, int Hq, int Hkv, int D, float eps, bool qk_norm,
                      bool q_tm, cudaStream_t s);
void qk_norm_rope_bwd(const bf16* dq, const bf16* dk, const bf16* dv, const bf16* kqv,
                      const bf16* qw, const bf16* kw, const float* cos_t, const float* sin_t,
                      const int32_t* pos, const float* rstd, bf16* dkqv, float* dqw, float* dkw,
                      int B, int S, int Hq, int Hkv, int D, bool qk_norm, bool q_tm,
                      bf16* dqw_out, bf16* dkw_out, int* ticket, cudaStream_t s);
// (with dqw_out/dkw_out: dqw is a zeroed [2D] accumulator slot, dkw == dqw + D)

void embedding_fwd(const int64_t* ids, const bf16* table, bf16* out, int64_t T, int H, int64_t V,
                   cudaStream_t s);
void embedding_bwd(const int64_t* ids, const bf16* dy, float* dtable, int64_t T, int H, int64_t V,
                   cudaStream_t s);
// Same from ids sorted ascending; order[p] = token row of sorted position p.
// H <= 1024.  dtable fp32 [V, H] (accumulated into).
void embedding_bwd_sorted(const int64_t* sorted_ids, const int64_t* order, const bf16* dy,
                          float* dtable, int64_t T, int H, int64_t V, cudaStream_t s);

// Cross-entropy from bf16 logits and per-(row, n-tile) (max, sumexp) partials.
// Writes loss[row] and overwrites logits with d(loss_sum*scale)/d(logits).
void ce_loss_grad(bf16* logits, const float* stats, int ntiles, const int64_t* targets,
                  float* loss, const float* scale, int64_t T, int V, int64_t ignore_index,
                  cudaStream_t s);

// Per-token routed expert scales: row_scale[t, e] = routed_scale * sum_j w_j [R[j, id_t] == e].
void route_scales(const int64_t* ids, const int64_t* table, const float* route_w, float* out,
                  int64_t T, int top_k, int64_t V, int E, float routed_scale, cudaStream_t s);

// Flat-buffer AdamW (torch.optim.AdamW semantics) with fp32 master weights;
// writes the bf16 compute copy.  clip (device scalar or nullptr) scales grads.
// hyper (device [lr, bc1, bc2] or nullptr) overrides lr/bc1/bc2, so a CUDA
// graph that captured the launch follows the schedule across replays.
void adamw_flat(float* p, float* m, float* v, const bf16* g, bf16* p_out, int64_t n, float lr,
                float beta1, float beta2, float eps, float wd, float bc1, float bc2,
                const float* clip, const float* hyper, cudaStream_t s);
// sumsq (+=) of a bf16 vector into *out (fp32, caller zeroes).
void sumsq_bf16(const bf16* g, int64_t n, float* out, cudaStream_t s);
// clip = min(1, max_norm / (sqrt(sumsq) + 1e-6)); norm = sqrt(sumsq).
void clip_coef(const float* sumsq, float max_norm, float* clip, float* norm, cudaStream_t s);

// Causal attention of ragged new-token queries q [N,Hq,D] over paged K/V pools
// [pages, page_size, Hkv, D]; page_table [num_seqs, max_pages], cu_q [num_seqs+1],
// kv_lens [num_seqs] (int32).  Writes out [N,Hq,D].  The KV range is split
// into `splits` ranges of `pages_per_split` pages (splits * pages_per_split >=
// max_pages); with splits > 1, ws_o [N*Hq*splits*D] and ws_lse [N*Hq*splits]
// (fp32) hold the partials.
int paged_attention(const bf16* q, const bf16* k_pool, const bf16* v_pool,
                    const int32_t* page_table, const int32_t* cu_q, const int32_t* kv_lens,
                    bf16* out, float* ws_o, float* ws_lse, int N, int num_seqs, int max_pages,
                    int Hq, int Hkv, int D, int page_size, int pages_per_split, int splits,
                    float scale, cudaStream_t s);
// RMSNorm (optional) + RoPE of the new tokens' q/k heads from kqv [N, (Hkv+Hq+Hkv)*D];
// q -> q_out [N,Hq,D], k and v -> their slots of one layer's pools [*, Hkv, D].
int paged_qkv_rope(const bf16* kqv, const bf16* qw, const bf16* kw, const float* cos_t,
                   const float* sin_t, const int64_t* pos, const int64_t* slots, bf16* q_out,
                   bf16* k_layer, bf16* v_layer, int N, int Hq, int Hkv, int D, float eps,
                   bool qk_norm, cudaStream_t s);
// KV split of paged_attention for N query tokens, Hkv heads and page tables
// `max_pages` wide (about eight CTAs per SM).
void paged_attention_split(int N, int Hkv, int max_kv, int num_sms, int* pages_per_split,
                           int* splits);

// Batched strided 2-D copies (pack.cu): dst(r, c) = src(r, c) for r < rows,
// c < cols, where a side's element offset is (r / div) * hi + (r % div) * lo
// + c * cs; src is fp32 (src_f32) or bf16, dst bf16.
constexpr int kMaxCopyJobs = 8;
struct CopyJob {
  const void* src = nullptr;
  bf16* dst = nullptr;
  int rows = 0, cols = 0;
  int s_div = 1, d_div = 1;
  int64_t s_hi = 0, s_lo = 0, s_cs = 1;
  int64_t d_hi = 0, d_lo = 0, d_cs = 1;
  int src_f32 = 0;
  int vec = 0;        // set by copy_jobs: unit column strides and 16-byte aligned rows
  int64_t unit0 = 0;  // set by copy_jobs: first work unit of this job
};
struct CopyJobs {
  CopyJob j[kMaxCopyJobs];
  int n = 0;
};
void copy_jobs(const CopyJobs& jobs, cudaStream_t s);

// Expert-contiguous routed experts (moe_grouped.cu).  routes int64 [k, T];
// rows_bound = moe_rows_bound(k*T, E) sorted rows (segments padded to 256).
int moe_rows_bound(int64_t n_assign, int E);
int moe_plan_launch(const int64_t* routes, int k, int64_t T, int E, const float* slot_w,
                    int* blk_hist, int* seg_start, int* tile_group, int* row_token,
                    float* row_weight, int* token_pos, cudaStream_t stream);
int moe_gather_launch(const void* src, const int* row_token, void* dst, int64_t rows, int H,
                      float scale, int num_sms, cudaStream_t stream);
int moe_combine_launch(const void* src, const int* token_pos, const void* base, void* out,
                       int64_t T, int H, int k, float scale, int num_sms, cudaStream_t stream);

}  // namespace cfb
