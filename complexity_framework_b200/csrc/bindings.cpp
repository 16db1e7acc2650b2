// Python bindings of the sm_100a kernels.  Every entry point validates shapes,
// dtypes, devices and alignment on the host and raises on violation: no silent
// fallback.  Kernels report device-side failures (bounded-wait timeouts,
// bounds checks) through a per-device error word read by check_errors().
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <vector>
#include <unordered_map>

#include "dist_fused.h"
#include "tp_fused.h"
#include "tp_decode.h"
#include "fsdp.h"
#include "ep_fused.h"
#include "flash.h"
#include "gemm_tc.h"
#include "kernels.h"

namespace {

std::mutex g_err_mu;
std::unordered_map<int, torch::Tensor> g_err;

int* err_ptr(int device) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  auto it = g_err.find(device);
  if (it == g_err.end()) {
    auto t = torch::zeros({4}, torch::dtype(torch::kInt32).device(torch::kCUDA, device));
    it = g_err.emplace(device, t).first;
  }
  return it->second.data_ptr<int>();
}

torch::Tensor error_buffer(int64_t device) {
  err_ptr(static_cast<int>(device));
  std::lock_guard<std::mutex> lk(g_err_mu);
  return g_err[static_cast<int>(device)];
}

int num_sms(int device) {
  static std::unordered_map<int, int> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
  cache[device] = v;
  return v;
}

void check_bf16_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16");
}

// Row-major 2-D view check: last stride 1, leading dim multiple of 8 elements,
// base 16-byte aligned (TMA requirements).
int64_t ld_of(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have unit inner stride");
  const int64_t ld = t.size(0) > 1 ? t.stride(0) : t.size(1);
  TORCH_CHECK(ld % 8 == 0, name, " leading dimension must be a multiple of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
  return ld;
}

void raise_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " launch failed with code ", rc,
              rc > 0 && rc < 1000 ? cudaGetErrorString(static_cast<cudaError_t>(rc)) : "");
}

// C[M,N] = epi(sum_k A(m,k) B(n,k)).  See gemm_tc.h for operand conventions.
static void build_gemm(cfb::GemmArgs& g, cfb::GemmEpi& ep, bool seg_a, bool seg_b, bool peer,
                       const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn, int64_t M,
          int64_t N, int64_t K, int64_t epi, const c10::optional<torch::Tensor>& out,
          const c10::optional<torch::Tensor>& residual, double alpha,
          const c10::optional<torch::Tensor>& gu, const c10::optional<torch::Tensor>& act,
          const c10::optional<torch::Tensor>& row_scale, int64_t shared_width,
          int64_t expert_width, int64_t n_experts, double shared_scale,
          const c10::optional<torch::Tensor>& stats, int64_t bn) {
  check_bf16_cuda(A, "A");
  check_bf16_cuda(B, "B");
  const c10::cuda::CUDAGuard guard(A.device());
  g.A = A.data_ptr();
  g.lda = ld_of(A, "A");
  g.a_mn = a_mn;
  g.B = B.data_ptr();
  g.ldb = ld_of(B, "B");
  g.b_mn = b_mn;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.epi = static_cast<int>(epi);
  g.bn = static_cast<int>(bn);
  g.num_sms = num_sms(A.get_device());
  TORCH_CHECK(N % 32 == 0, "gemm: N must be a multiple of 32");
  // operand extents
  if (!seg_a) {
    if (!a_mn) {
      TORCH_CHECK(A.size(0) >= M && A.size(1) >= K, "gemm: A too small");
    } else {
      TORCH_CHECK(A.size(0) >= K && A.size(1) >= M, "gemm: A too small");
    }
  }
  if (!seg_b) {
    if (!b_mn) {
      TORCH_CHECK(B.size(0) >= N && B.size(1) >= K, "gemm: B too small");
    } else {
      TORCH_CHECK(B.size(0) >= K && B.size(1) >= N, "gemm: B too small");
    }
  }

  ep.alpha = static_cast<float>(alpha);
  if (epi == cfb::EPI_SWIGLU_FWD) {
    TORCH_CHECK(gu.has_value() && act.has_value(), "swiglu fwd needs gu and act");
    check_bf16_cuda(*gu, "gu");
    check_bf16_cuda(*act, "act");
    TORCH_CHECK(gu->size(0) >= M && gu->size(1) >= N, "gu too small");
    TORCH_CHECK(act->size(0) >= M && act->size(1) >= N / 2, "act too small");
    TORCH_CHECK(N % (2 * cfb::kSwigluBlock) == 0, "swiglu fwd: N must be a multiple of 256");
    ep.gu = reinterpret_cast<__nv_bfloat16*>(gu->data_ptr());
    ep.ldgu = ld_of(*gu, "gu");
    ep.act = reinterpret_cast<__nv_bfloat16*>(act->data_ptr());
    ep.ldact = ld_of(*act, "act");
  } else {
    TORCH_CHECK(out.has_value(), "gemm needs out");
    TORCH_CHECK(out->is_cuda(), "out must be CUDA");
    const bool f32 = epi == cfb::EPI_F32 || epi == cfb::EPI_F32_ACC ||
                     epi == cfb::EPI_F32_ATOMIC || epi == cfb::EPI_PEER_STORE;
    TORCH_CHECK(out->scalar_type() == (f32 ? torch::kFloat32 : torch::kBFloat16),
                "out dtype mismatch for epilogue");
    TORCH_CHECK(out->dim() == 2 && out->stride(1) == 1, "out must be row-major 2-D");
    ep.c = out->data_ptr();
    ep.ldc = out->size(0) > 1 ? out->stride(0) : out->size(1);
    TORCH_CHECK(ep.ldc % 8 == 0, "out leading dim must be a multiple of 8");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(ep.c) % 16 == 0, "out must be 16-byte aligned");
    if (epi == cfb::EPI_SWIGLU_BWD) {
      TORCH_CHECK(out->size(0) >= M && out->size(1) >= 2 * N, "d(gu) too small");
      TORCH_CHECK(N % cfb::kSwigluBlock == 0, "swiglu bwd: N must be a multiple of 128");
      TORCH_CHECK(gu.has_value(), "swiglu bwd needs gu");
      check_bf16_cuda(*gu, "gu");
      ep.gu = reinterpret_cast<__nv_bfloat16*>(gu->data_ptr());
      ep.ldgu = ld_of(*gu, "gu");
    } else if (!peer) {
      TORCH_CHECK(out->size(0) >= M && out->size(1) >= N, "out too small");
    }
  }
  if (epi == cfb::EPI_RESID) {
    TORCH_CHECK(residual.has_value(), "residual epilogue needs residual");
    check_bf16_cuda(*residual, "residual");
    TORCH_CHECK(residual->size(0) >= M && residual->size(1) >= N, "residual too small");
    ep.r = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    ep.ldr = ld_of(*residual, "residual");
  }
  if (epi == cfb::EPI_SWIGLU_FWD || epi == cfb::EPI_SWIGLU_BWD) {
    ep.shared_width = static_cast<int>(shared_width);
    ep.expert_width = static_cast<int>(expert_width > 0 ? expert_width : 1);
    ep.n_experts = static_cast<int>(n_experts);
    ep.shared_scale = static_cast<float>(shared_scale);
    const int64_t act_width = epi == cfb::EPI_SWIGLU_FWD ? N / 2 : N;
    TORCH_CHECK(shared_width % 32 == 0 && (n_experts == 0 || expert_width % 32 == 0),
                "swiglu widths must be multiples of 32");
    TORCH_CHECK(shared_width + n_experts * expert_width == act_width,
                "swiglu: shared_width + n_experts*expert_width must equal activation width");
    if (n_experts > 0) {
      TORCH_CHECK(row_scale.has_value(), "routed experts need row_scale");
      TORCH_CHECK(row_scale->scalar_type() == torch::kFloat32 && row_scale->is_contiguous(),
                  "row_scale must be contiguous fp32");
      TORCH_CHECK(row_scale->numel() >= M * n_experts, "row_scale too small");
      ep.row_scale = row_scale->data_ptr<float>();
    }
  }
  if (epi == cfb::EPI_CE_STATS) {
    TORCH_CHECK(stats.has_value() && stats->scalar_type() == torch::kFloat32 &&
                    stats->is_contiguous(),
                "ce stats epilogue needs contiguous fp32 stats");
    TORCH_CHECK(bn == 0 || bn == 256, "ce stats epilogue runs with 256-column tiles");
    g.bn = 256;
    TORCH_CHECK(stats->numel() >= M * 2 * ((N + 255) / 256) * 2, "stats too small");
    ep.stats = stats->data_ptr<float>();
  }
}

void gemm(const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn, int64_t M,
          int64_t N, int64_t K, int64_t epi, const c10::optional<torch::Tensor>& out,
          const c10::optional<torch::Tensor>& residual, double alpha,
          const c10::optional<torch::Tensor>& gu, const c10::optional<torch::Tensor>& act,
          const c10::optional<torch::Tensor>& row_scale, int64_t shared_width,
          int64_t expert_width, int64_t n_experts, double shared_scale,
          const c10::optional<torch::Tensor>& stats, int64_t bn) {
  cfb::GemmArgs g;
  cfb::GemmEpi ep;
  build_gemm(g, ep, false, false, false, A, a_mn, B, b_mn, M, N, K, epi, out, residual, alpha, gu,
             act, row_scale, shared_width, expert_width, n_experts, shared_scale, stats, bn);
  const int rc = cfb::gemm_tc_launch(g, ep, at::cuda::getCurrentCUDAStream(),
                                     err_ptr(A.get_device()));
  raise_rc(rc, "gemm");
}

// Tensor-parallel GEMMs: all-gather fused into the operand loads (segments of
// A or B in peer memory) and reduce-scatter by peer stores of fp32 partials.
void gemm_dist(const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn, int64_t M,
               int64_t N, int64_t K, int64_t epi, const c10::optional<torch::Tensor>& out,
               const c10::optional<torch::Tensor>& gu, const c10::optional<torch::Tensor>& act,
               const c10::optional<torch::Tensor>& row_scale, int64_t shared_width,
               int64_t expert_width, int64_t n_experts, double shared_scale,
               const std::vector<int64_t>& a_seg, int64_t a_seg_rows,
               const std::vector<int64_t>& b_seg, int64_t b_seg_rows,
               const std::vector<int64_t>& peer_c, int64_t peer_rows,
               const std::vector<int64_t>& pads, int64_t rank, int64_t round, int64_t epoch,
               int64_t role, bool signal, const std::vector<int64_t>& ag_src,
               const c10::optional<torch::Tensor>& ag_flags, int64_t ag_rows, int64_t ag_epoch) {
  TORCH_CHECK(a_seg.size() <= static_cast<size_t>(cfb::kMaxSeg) &&
                  b_seg.size() <= static_cast<size_t>(cfb::kMaxSeg) &&
                  peer_c.size() <= static_cast<size_t>(cfb::kMaxSeg) &&
                  pads.size() <= static_cast<size_t>(cfb::kMaxSeg),
              "at most 8 ranks");
  const bool peer = epi == cfb::EPI_PEER_STORE;
  cfb::GemmArgs g;
  cfb::GemmEpi ep;
  build_gemm(g, ep, !a_seg.empty(), !b_seg.empty(), peer, A, a_mn, B, b_mn, M, N, K, epi, out,
             c10::nullopt, 1.0, gu, act, row_scale, shared_width, expert_width, n_experts,
             shared_scale, c10::nullopt, 0);
  g.a_nseg = static_cast<int>(a_seg.size());
  g.a_seg_rows = a_seg_rows;
  for (size_t i = 0; i < a_seg.size(); ++i) g.A_seg[i] = reinterpret_cast<const void*>(a_seg[i]);
  g.b_nseg = static_cast<int>(b_seg.size());
  g.b_seg_rows = b_seg_rows;
  for (size_t i = 0; i < b_seg.size(); ++i) g.B_seg[i] = reinterpret_cast<const void*>(b_seg[i]);
  if (peer) {
    TORCH_CHECK(peer_c.size() == pads.size() && peer_rows > 0, "peer store needs peer buffers");
    for (size_t i = 0; i < peer_c.size(); ++i) ep.peer_c[i] = reinterpret_cast<float*>(peer_c[i]);
    ep.peer_rows = peer_rows;
  }
  ep.sync.world = static_cast<int>(pads.size());
  for (size_t i = 0; i < pads.size(); ++i) ep.sync.pad[i] = reinterpret_cast<int*>(pads[i]);
  ep.sync.rank = static_cast<int>(rank);
  ep.sync.round = static_cast<int>(round);
  ep.sync.epoch = static_cast<int>(epoch);
  ep.sync.role = static_cast<int>(role);
  ep.sync.signal = signal ? 1 : 0;
  if (!ag_src.empty()) {
    // fused all-gather: A is this rank's full gathered buffer [world*ag_rows, K]
    TORCH_CHECK(ag_src.size() == pads.size() && !a_mn && a_seg.empty(),
                "fused all-gather: one source per rank, K-major A");
    TORCH_CHECK(ag_rows % 128 == 0 && ag_rows * static_cast<int64_t>(pads.size()) == M,
                "fused all-gather: rows per rank must be a multiple of 128 and sum to M");
    TORCH_CHECK(ag_flags.has_value() && ag_flags->scalar_type() == torch::kInt32 &&
                    ag_flags->numel() >= M / 128,
                "fused all-gather needs int32 flags, one per 128 rows");
    TORCH_CHECK(A.size(0) >= M && A.stride(0) == K && K % 8 == 0,
                "fused all-gather: A must be the contiguous gathered buffer");
    for (size_t i = 0; i < ag_src.size(); ++i)
      ep.ag.src[i] = reinterpret_cast<const __nv_bfloat16*>(ag_src[i]);
    ep.ag.dst = reinterpret_cast<__nv_bfloat16*>(A.data_ptr());
    ep.ag.flags = ag_flags->data_ptr<int>();
    ep.ag.rows = static_cast<int>(ag_rows);
    ep.ag.cols = static_cast<int>(K);
    ep.ag.epoch = static_cast<int>(ag_epoch);
    ep.ag.active = 1;
    g.bn = 256;
  }
  const int rc = cfb::gemm_tc_launch(g, ep, at::cuda::getCurrentCUDAStream(),
                                     err_ptr(A.get_device()));
  raise_rc(rc, "gemm_dist");
}

static cfb::TpSync make_tp_sync(const std::vector<int64_t>& pads, int64_t rank, int64_t round,
                                 int64_t epoch) {
  TORCH_CHECK(!pads.empty() && pads.size() <= 8, "1..8 ranks");
  cfb::TpSync sy{};
  for (size_t i = 0; i < pads.size(); ++i) sy.pad[i] = reinterpret_cast<int*>(pads[i]);
  sy.world = static_cast<int>(pads.size());
  sy.rank = static_cast<int>(rank);
  sy.round = static_cast<int>(round);
  sy.epoch = static_cast<int>(epoch);
  return sy;
}

// Sum, for this rank's rows, the world bf16 partial products (+ residual) into bf16 out.
void tp_rs_finish(const std::vector<int64_t>& parts, int64_t rows, int64_t n, int64_t ld,
                  const c10::optional<torch::Tensor>& residual, torch::Tensor& out,
                  const std::vector<int64_t>& pads, int64_t rank, int64_t round, int64_t epoch) {
  TORCH_CHECK(parts.size() == pads.size(), "one partial buffer per rank");
  check_bf16_cuda(out, "out");
  TORCH_CHECK(out.dim() == 2 && out.size(0) >= rows && out.size(1) >= n && out.stride(1) == 1,
              "out too small");
  const __nv_bfloat16* r = nullptr;
  int64_t ldr = 0;
  if (residual.has_value()) {
    check_bf16_cuda(*residual, "residual");
    TORCH_CHECK(residual->stride(-1) == 1 && residual->stride(0) % 8 == 0, "residual layout");
    r = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    ldr = residual->stride(0);
  }
  cfb::TpPartials pp{};
  for (size_t i = 0; i < parts.size(); ++i)
    pp.part[i] = reinterpret_cast<const __nv_bfloat16*>(parts[i]);
  const c10::cuda::CUDAGuard guard(out.device());
  const int rc = cfb::tp_rs_finish(pp, rows, static_cast<int>(n), ld, r, ldr,
                                   reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                   out.stride(0), make_tp_sync(pads, rank, round, epoch),
                                   num_sms(out.get_device()),
                                   at::cuda::getCurrentCUDAStream(), err_ptr(out.get_device()));
  raise_rc(rc, "tp_rs_finish");
}

void tp_barrier(const std::vector<int64_t>& pads, int64_t rank, int64_t round, int64_t epoch,
                int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  const int rc = cfb::tp_barrier(make_tp_sync(pads, rank, round, epoch),
                                 at::cuda::getCurrentCUDAStream(),
                                 err_ptr(static_cast<int>(device)));
  raise_rc(rc, "tp_barrier");
}

// ZeRO-3: gather every rank's bf16 shard of a unit into this rank's full buffer.
void fsdp_gather(const std::vector<int64_t>& shards, const std::vector<int64_t>& pads,
                 int64_t rank, torch::Tensor& dst, int64_t shard, int64_t round,
                 int64_t epoch) {
  check_bf16_cuda(dst, "dst");
  TORCH_CHECK(dst.is_contiguous(), "dst must be contiguous");
  TORCH_CHECK(!shards.empty() && shards.size() <= cfb::kFsdpMaxRanks &&
                  pads.size() == shards.size(), "1..8 ranks with one pad each");
  TORCH_CHECK(dst.numel() >= shard * static_cast<int64_t>(shards.size()), "dst too small");
  TORCH_CHECK(round >= 0 && round < 4, "pads hold 4 rounds");
  cfb::FsdpPeers pp{};
  pp.world = static_cast<int>(shards.size());
  pp.rank = static_cast<int>(rank);
  for (size_t i = 0; i < shards.size(); ++i) {
    pp.shard[i] = reinterpret_cast<const __nv_bfloat16*>(shards[i]);
    pp.pad[i] = reinterpret_cast<int*>(pads[i]);
  }
  const int dev = dst.get_device();
  const c10::cuda::CUDAGuard guard(dst.device());
  const int rc = cfb::fsdp_gather(pp, reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), shard,
                                  static_cast<int>(round), static_cast<int>(epoch), num_sms(dev),
                                  at::cuda::getCurrentCUDAStream(), err_ptr(dev));
  raise_rc(rc, "fsdp_gather");
}

// out = residual + sum over ranks of their partial buffers (decode tensor parallelism).
void tp_allreduce(const std::vector<int64_t>& bufs, const std::vector<int64_t>& pads,
                  int64_t mc, int64_t rank, const c10::optional<torch::Tensor>& residual,
                  torch::Tensor& out, torch::Tensor& epoch, torch::Tensor& ticket) {
  check_bf16_cuda(out, "out");
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  TORCH_CHECK(!bufs.empty() && bufs.size() <= cfb::kTpMaxRanks && pads.size() == bufs.size(),
              "1..8 ranks with one pad each");
  TORCH_CHECK(epoch.is_cuda() && epoch.scalar_type() == torch::kInt32 && ticket.is_cuda() &&
                  ticket.scalar_type() == torch::kInt32, "epoch / ticket: int32 CUDA");
  cfb::TpArPtrs pp{};
  pp.world = static_cast<int>(bufs.size());
  pp.rank = static_cast<int>(rank);
  for (size_t i = 0; i < bufs.size(); ++i) {
    pp.buf[i] = reinterpret_cast<const __nv_bfloat16*>(bufs[i]);
    pp.pad[i] = reinterpret_cast<int*>(pads[i]);
  }
  pp.mc = reinterpret_cast<const __nv_bfloat16*>(mc);
  const __nv_bfloat16* r = nullptr;
  if (residual.has_value()) {
    check_bf16_cuda(*residual, "residual");
    TORCH_CHECK(residual->is_contiguous() && residual->numel() == out.numel(),
                "residual must be contiguous like out");
    r = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  const int dev = out.get_device();
  const c10::cuda::CUDAGuard guard(out.device());
  const int rc = cfb::tp_allreduce(pp, r, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                   out.numel(), epoch.data_ptr<int>(), ticket.data_ptr<int>(),
                                   num_sms(dev), at::cuda::getCurrentCUDAStream(), err_ptr(dev));
  raise_rc(rc, "tp_allreduce");
}

// out[i] = residual[i] + sum_j w[i,j] * rows of peers' buffers (EP dispatch / combine).
void ep_gather_combine(const std::vector<int64_t>& srcs, const torch::Tensor& idx,
                       const c10::optional<torch::Tensor>& w, int64_t stride,
                       const c10::optional<torch::Tensor>& residual, torch::Tensor& out,
                       const std::vector<int64_t>& pads, int64_t rank, int64_t round,
                       int64_t epoch) {
  check_bf16_cuda(out, "out");
  TORCH_CHECK(out.dim() == 2 && out.is_contiguous(), "out must be contiguous [rows, H]");
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == torch::kInt32 && idx.is_contiguous() &&
                  idx.dim() == 2 && idx.size(0) == out.size(0),
              "idx must be int32 [rows, k]");
  TORCH_CHECK(!srcs.empty() && srcs.size() <= 8 && pads.size() <= 8, "1..8 ranks");
  const int k = static_cast<int>(idx.size(1));
  const float* wp = nullptr;
  if (w.has_value()) {
    TORCH_CHECK(w->scalar_type() == torch::kFloat32 && w->is_contiguous() &&
                    w->numel() == idx.numel(),
                "w must be fp32 like idx");
    wp = w->data_ptr<float>();
  }
  const __nv_bfloat16* r = nullptr;
  if (residual.has_value()) {
    check_bf16_cuda(*residual, "residual");
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == out.sizes(), "residual shape");
    r = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  cfb::EpSources es{};
  for (size_t i = 0; i < srcs.size(); ++i)
    es.p[i] = reinterpret_cast<const __nv_bfloat16*>(srcs[i]);
  cfb::EpSync sy{};
  for (size_t i = 0; i < pads.size(); ++i) sy.pad[i] = reinterpret_cast<int*>(pads[i]);
  sy.world = static_cast<int>(pads.size());
  sy.world_srcs = static_cast<int>(srcs.size());
  sy.rank = static_cast<int>(rank);
  sy.round = static_cast<int>(round);
  sy.epoch = static_cast<int>(epoch);
  const c10::cuda::CUDAGuard guard(out.device());
  const int rc = cfb::ep_gather_combine(es, idx.data_ptr<int>(), wp, out.size(0),
                                        static_cast<int>(out.size(1)), stride, r,
                                        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), k, sy,
                                        num_sms(out.get_device()),
                                        at::cuda::getCurrentCUDAStream(),
                                        err_ptr(out.get_device()));
  raise_rc(rc, "ep_gather_combine");
}

// Grouped GEMM: gemm() plus the group tables of GemmGroups (gemm_tc.h).
// mode 1: tile_group int32 [M / 256], b_stride; mode 2: k_start int32 [groups + 1],
// c_stride (fp32 atomic epilogue only).
void gemm_grouped(const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn, int64_t M,
                  int64_t N, int64_t K, int64_t epi, const c10::optional<torch::Tensor>& out,
                  const c10::optional<torch::Tensor>& gu, const c10::optional<torch::Tensor>& act,
                  const c10::optional<torch::Tensor>& row_scale, int64_t expert_width,
                  int64_t mode, const c10::optional<torch::Tensor>& tile_group,
                  const c10::optional<torch::Tensor>& k_start, int64_t groups, int64_t b_stride,
                  int64_t c_stride, double alpha) {
  cfb::GemmArgs g;
  cfb::GemmEpi ep;
  const bool swiglu = epi == cfb::EPI_SWIGLU_FWD || epi == cfb::EPI_SWIGLU_BWD;
  build_gemm(g, ep, false, false, false, A, a_mn, B, b_mn, M, N, K, epi, out, c10::nullopt, alpha,
             gu, act, row_scale, 0, swiglu ? expert_width : 0, swiglu ? 1 : 0, 1.0, c10::nullopt,
             0);
  TORCH_CHECK(groups > 0, "gemm_grouped: groups must be positive");
  ep.grp.mode = static_cast<int>(mode);
  ep.grp.ngroups = static_cast<int>(groups);
  if (mode == 1) {
    TORCH_CHECK(tile_group.has_value() && tile_group->scalar_type() == torch::kInt32 &&
                    tile_group->is_contiguous() && tile_group->is_cuda() &&
                    tile_group->numel() >= M / 256,
                "mode 1 needs int32 tile_group [M / 256]");
    TORCH_CHECK(M % 256 == 0, "mode 1: M must be a multiple of 256");
    TORCH_CHECK(b_stride > 0, "mode 1 needs b_stride");
    TORCH_CHECK(b_mn ? B.size(0) >= groups * b_stride : B.size(0) >= groups * b_stride,
                "gemm_grouped: B holds fewer than groups * b_stride rows");
    ep.grp.tile_group = tile_group->data_ptr<int>();
    ep.grp.b_stride = b_stride;
  } else if (mode == 2) {
    TORCH_CHECK(k_start.has_value() && k_start->scalar_type() == torch::kInt32 &&
                    k_start->is_contiguous() && k_start->is_cuda() &&
                    k_start->numel() >= groups + 1,
                "mode 2 needs int32 k_start [groups + 1]");
    TORCH_CHECK(epi == cfb::EPI_F32_ATOMIC && a_mn && b_mn,
                "mode 2 is the fp32 atomic weight-gradient GEMM with MN-major operands");
    TORCH_CHECK(out->size(0) >= groups * c_stride && c_stride >= M, "mode 2: out too small");
    ep.grp.k_start = k_start->data_ptr<int>();
    ep.grp.c_stride = c_stride;
  } else {
    TORCH_CHECK(false, "gemm_grouped: mode must be 1 or 2");
  }
  const int rc = cfb::gemm_tc_launch(g, ep, at::cuda::getCurrentCUDAStream(),
                                     err_ptr(A.get_device()));
  raise_rc(rc, "gemm_grouped");
}

// Expert-contiguous plan of routes int64 [k, T] over E experts with per-slot
// weights slot_w fp32 [k]: (seg_start [E+1], tile_group [R/256], row_token [R],
// row_weight [R], token_pos [k*T]) with R = moe_rows_bound(k*T, E).
std::vector<torch::Tensor> moe_plan(const torch::Tensor& routes, int64_t E,
                                    const torch::Tensor& slot_w) {
  TORCH_CHECK(routes.is_cuda() && routes.scalar_type() == torch::kInt64 && routes.dim() == 2 &&
                  routes.is_contiguous(),
              "routes must be contiguous int64 [k, T] on CUDA");
  TORCH_CHECK(slot_w.is_cuda() && slot_w.scalar_type() == torch::kFloat32 &&
                  slot_w.numel() == routes.size(0),
              "slot_w must be fp32 [k] on CUDA");
  const c10::cuda::CUDAGuard guard(routes.device());
  const int64_t k = routes.size(0), T = routes.size(1);
  const int64_t R = cfb::moe_rows_bound(k * T, static_cast<int>(E));
  auto i32 = torch::dtype(torch::kInt32).device(routes.device());
  const int64_t nblk = (k * T + 1023) / 1024;
  auto blk = torch::empty({nblk * E}, i32);
  auto seg = torch::empty({E + 1}, i32);
  auto tiles = torch::empty({R / 256}, i32);
  auto row_token = torch::empty({R}, i32);
  auto row_weight = torch::empty({R}, torch::dtype(torch::kFloat32).device(routes.device()));
  auto token_pos = torch::empty({k * T}, i32);
  const int rc = cfb::moe_plan_launch(routes.data_ptr<int64_t>(), static_cast<int>(k), T,
                                      static_cast<int>(E), slot_w.data_ptr<float>(),
                                      blk.data_ptr<int>(), seg.data_ptr<int>(),
                                      tiles.data_ptr<int>(), row_token.data_ptr<int>(),
                                      row_weight.data_ptr<float>(), token_pos.data_ptr<int>(),
                                      at::cuda::getCurrentCUDAStream());
  raise_rc(rc, "moe_plan");
  return {seg, tiles, row_token, row_weight, token_pos};
}

// dst [R, H] = scale * src[row_token] (zero rows where row_token < 0)
torch::Tensor moe_gather(const torch::Tensor& src, const torch::Tensor& row_token, double scale) {
  check_bf16_cuda(src, "src");
  TORCH_CHECK(src.dim() == 2 && src.is_contiguous(), "src must be contiguous [T, H]");
  TORCH_CHECK(row_token.scalar_type() == torch::kInt32 && row_token.is_contiguous(),
              "row_token must be contiguous int32");
  const c10::cuda::CUDAGuard guard(src.device());
  auto dst = torch::empty({row_token.numel(), src.size(1)}, src.options());
  const int rc = cfb::moe_gather_launch(src.data_ptr(), row_token.data_ptr<int>(), dst.data_ptr(),
                                        row_token.numel(), static_cast<int>(src.size(1)),
                                        static_cast<float>(scale), num_sms(src.get_device()),
                                        at::cuda::getCurrentCUDAStream());
  raise_rc(rc, "moe_gather");
  return dst;
}

// out [T, H] = base + scale * sum_j src[token_pos[j*T + t]]
torch::Tensor moe_combine(const torch::Tensor& src, const torch::Tensor& token_pos, int64_t k,
                          double scale, const c10::optional<torch::Tensor>& base) {
  check_bf16_cuda(src, "src");
  TORCH_CHECK(src.dim() == 2 && src.is_contiguous(), "src must be contiguous [R, H]");
  TORCH_CHECK(token_pos.scalar_type() == torch::kInt32 && token_pos.is_contiguous() &&
                  token_pos.numel() % k == 0,
              "token_pos must be contiguous int32 [k*T]");
  const int64_t T = token_pos.numel() / k, H = src.size(1);
  if (base.has_value()) {
    check_bf16_cuda(*base, "base");
    TORCH_CHECK(base->is_contiguous() && base->numel() == T * H, "base must be [T, H]");
  }
  const c10::cuda::CUDAGuard guard(src.device());
  auto out = torch::empty({T, H}, src.options());
  const int rc = cfb::moe_combine_launch(src.data_ptr(), token_pos.data_ptr<int>(),
                                         base.has_value() ? base->data_ptr() : nullptr,
                                         out.data_ptr(), T, static_cast<int>(H),
                                         static_cast<int>(k), static_cast<float>(scale),
                                         num_sms(src.get_device()),
                                         at::cuda::getCurrentCUDAStream());
  raise_rc(rc, "moe_combine");
  return out;
}

// [B, H, S, D] bf16 view with a contiguous last dim and 16-byte aligned rows
// (TMA requirements) -> strided descriptor.
cfb::Bhsd bhsd_of(const torch::Tensor& t, const char* name) {
  check_bf16_cuda(t, name);
  TORCH_CHECK(t.dim() == 4, name, " must be [B, H, S, D]");
  TORCH_CHECK(t.stride(3) == 1, name, " must have a contiguous last dimension");
  for (int i = 0; i < 3; ++i)
    TORCH_CHECK(t.size(i) == 1 || t.stride(i) % 8 == 0, name,
                " strides must be multiples of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
  cfb::Bhsd d;
  d.p = t.data_ptr();
  d.sb = t.stride(0);
  d.sh = t.stride(1);
  d.ss = t.stride(2);
  return d;
}

// Causal/full attention forward; q [B,Hq,S,D] and k/v [B,Hkv,S,D] views (any
// strides, last dim contiguous); writes out [B,S,Hq*D] and lse [B,Hq,S].
void flash_attn_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                    torch::Tensor& out, torch::Tensor& lse, double scale, bool causal) {
  const cfb::Bhsd dq = bhsd_of(q, "q"), dk = bhsd_of(k, "k"), dv = bhsd_of(v, "v");
  check_bf16_cuda(out, "out");
  TORCH_CHECK(out.is_contiguous(), "flash_attn_fwd: out must be contiguous");
  TORCH_CHECK(v.sizes() == k.sizes(), "k/v shapes differ");
  const int64_t B = q.size(0), Hq = q.size(1), S = q.size(2), D = q.size(3), Hkv = k.size(1);
  TORCH_CHECK(k.size(0) == B && k.size(2) == S && k.size(3) == D, "k shape");
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TORCH_CHECK(out.numel() == B * S * Hq * D, "out size");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.is_contiguous() &&
                  lse.numel() == B * Hq * S,
              "lse must be fp32 [B,Hq,S]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int rc = cfb::flash_fwd_launch(dq, dk, dv, out.data_ptr(), lse.data_ptr<float>(), B, Hq,
                                       Hkv, S, D, static_cast<float>(scale), causal,
                                       at::cuda::getCurrentCUDAStream(), err_ptr(q.get_device()));
  raise_rc(rc, "flash_attn_fwd");
}

// Backward of flash_attn_fwd.  o, dout, dq: [B,Hq,S,D] views (the token-major
// [B,S,Hq*D] output seen through a transposed view is fine); dk, dv like k.
void flash_attn_bwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                    const torch::Tensor& o, const torch::Tensor& lse, const torch::Tensor& dout,
                    torch::Tensor& dq, torch::Tensor& dk, torch::Tensor& dv, double scale,
                    bool causal) {
  const cfb::Bhsd bq = bhsd_of(q, "q"), bk = bhsd_of(k, "k"), bv = bhsd_of(v, "v");
  const cfb::Bhsd bo = bhsd_of(o, "o"), bdo = bhsd_of(dout, "dout"), bdq = bhsd_of(dq, "dq");
  const cfb::Bhsd bdk = bhsd_of(dk, "dk"), bdv = bhsd_of(dv, "dv");
  const int64_t B = q.size(0), Hq = q.size(1), S = q.size(2), D = q.size(3), Hkv = k.size(1);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be a multiple of Hkv");
  TORCH_CHECK(k.sizes() == v.sizes() && dk.sizes() == k.sizes() && dv.sizes() == k.sizes() &&
                  k.size(0) == B && k.size(2) == S && k.size(3) == D,
              "k/v/dk/dv must be [B,Hkv,S,D]");
  TORCH_CHECK(o.sizes() == q.sizes() && dout.sizes() == q.sizes() && dq.sizes() == q.sizes(),
              "o/dout/dq must be [B,Hq,S,D]");
  TORCH_CHECK(dk.strides() == dv.strides(), "dk and dv must share strides");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.is_contiguous() &&
                  lse.numel() == B * Hq * S,
              "lse must be fp32 [B,Hq,S]");
  const c10::cuda::CUDAGuard guard(q.device());
  auto work = torch::empty({cfb::flash_bwd_workspace_floats(B, Hq, S, D)},
                           torch::dtype(torch::kFloat32).device(q.device()));
  const int rc = cfb::flash_bwd_launch(bq, bk, bv, bo, bdo, lse.data_ptr<float>(), bdq, bdk, bdv,
                                       B, Hq, Hkv, S, D, static_cast<float>(scale), causal,
                                       work.data_ptr<float>(), at::cuda::getCurrentCUDAStream(),
                                       err_ptr(q.get_device()));
  raise_rc(rc, "flash_attn_bwd");
}

cfb::PeerPtrs make_peers(const std::vector<int64_t>& grad, const std::vector<int64_t>& param,
                         const std::vector<int64_t>& pad, const std::vector<int64_t>& slots,
                         int64_t rank) {
  const size_t P = grad.size();
  TORCH_CHECK(P >= 1 && P <= static_cast<size_t>(cfb::kMaxRanks), "1..8 ranks supported");
  TORCH_CHECK(param.size() == P && pad.size() == P && slots.size() == P, "peer pointer lists");
  cfb::PeerPtrs pp{};
  for (size_t i = 0; i < P; ++i) {
    pp.grad[i] = reinterpret_cast<const __nv_bfloat16*>(grad[i]);
    pp.param[i] = reinterpret_cast<__nv_bfloat16*>(param[i]);
    pp.pad[i] = reinterpret_cast<int*>(pad[i]);
    pp.slots[i] = reinterpret_cast<float*>(slots[i]);
  }
  pp.world = static_cast<int>(P);
  pp.rank = static_cast<int>(rank);
  return pp;
}

// Reduce this rank's shard of the flat gradients of all peers (NVLink loads).
void dp_reduce_shard(const std::vector<int64_t>& grad, const std::vector<int64_t>& param,
                     const std::vector<int64_t>& pad, const std::vector<int64_t>& slots,
                     int64_t rank, int64_t lo, int64_t n, torch::Tensor& gs,
                     torch::Tensor& sumsq_local, torch::Tensor& ticket, int64_t epoch,
                     bool publish, const c10::optional<torch::Tensor>& epoch_dev) {
  TORCH_CHECK(gs.is_cuda() && gs.scalar_type() == torch::kBFloat16 && gs.numel() >= n,
              "gs must be this rank's bf16 gradient shard");
  const c10::cuda::CUDAGuard guard(gs.device());
  const auto pp = make_peers(grad, param, pad, slots, rank);
  const int rc = cfb::fused_reduce_shard(pp, lo, n,
                                         reinterpret_cast<__nv_bfloat16*>(gs.data_ptr()),
                                         sumsq_local.data_ptr<float>(), ticket.data_ptr<int>(),
                                         static_cast<int>(epoch),
                                         epoch_dev.has_value() ? epoch_dev->data_ptr<int>() : nullptr,
                                         publish, num_sms(gs.get_device()),
                                         at::cuda::getCurrentCUDAStream(), err_ptr(gs.get_device()));
  raise_rc(rc, "dp_reduce_shard");
}

// AdamW on the shard and store the new bf16 parameters into every peer.
void dp_adamw_shard(const std::vector<int64_t>& grad, const std::vector<int64_t>& param,
                    const std::vector<int64_t>& pad, const std::vector<int64_t>& slots,
                    int64_t rank, int64_t lo, int64_t n, torch::Tensor& master, torch::Tensor& m,
                    torch::Tensor& v, const torch::Tensor& gs, double lr, double b1, double b2,
                    double eps, double wd, double bc1, double bc2, double max_norm,
                    torch::Tensor& norm_out, torch::Tensor& ticket, int64_t epoch,
                    const c10::optional<torch::Tensor>& epoch_dev,
                    const c10::optional<torch::Tensor>& hyper) {
  if (hyper.has_value())
    TORCH_CHECK(hyper->is_cuda() && hyper->scalar_type() == torch::kFloat32 &&
                    hyper->is_contiguous() && hyper->numel() >= 3,
                "hyper must be contiguous fp32 (lr, bc1, bc2) on CUDA");
  for (const auto* t : {&master, &m, &v}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->numel() >= n,
                "fp32 optimizer shard");
  }
  const c10::cuda::CUDAGuard guard(master.device());
  const auto pp = make_peers(grad, param, pad, slots, rank);
  const int rc = cfb::fused_adamw_shard(
      pp, lo, n, master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      reinterpret_cast<const __nv_bfloat16*>(gs.data_ptr()), static_cast<float>(lr),
      static_cast<float>(b1),
      static_cast<float>(b2), static_cast<float>(eps), static_cast<float>(wd),
      static_cast<float>(bc1), static_cast<float>(bc2), static_cast<float>(max_norm),
      norm_out.data_ptr<float>(), ticket.data_ptr<int>(), static_cast<int>(epoch),
      epoch_dev.has_value() ? epoch_dev->data_ptr<int>() : nullptr,
      hyper.has_value() ? hyper->data_ptr<float>() : nullptr,
      num_sms(master.get_device()), at::cuda::getCurrentCUDAStream(), err_ptr(master.get_device()));
  raise_rc(rc, "dp_adamw_shard");
}

int64_t gemm_choose_bn(int64_t M, int64_t N, int64_t device) {
  return cfb::choose_bn(static_cast<int>(M), static_cast<int>(N), num_sms(static_cast<int>(device)));
}

}  // namespace

void register_elementwise(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("error_buffer", &error_buffer);
  m.def("gemm_dist", &gemm_dist);
  m.def("tp_rs_finish", &tp_rs_finish);
  m.def("tp_barrier", &tp_barrier);
  m.def("tp_allreduce", &tp_allreduce);
  m.def("fsdp_gather", &fsdp_gather);
  m.def("ep_gather_combine", &ep_gather_combine);
  m.def("gemm", &gemm, "tcgen05 GEMM with fused epilogues", py::arg("A"), py::arg("a_mn"),
        py::arg("B"), py::arg("b_mn"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi"),
        py::arg("out") = py::none(), py::arg("residual") = py::none(), py::arg("alpha") = 1.0,
        py::arg("gu") = py::none(), py::arg("act") = py::none(),
        py::arg("row_scale") = py::none(), py::arg("shared_width") = 0,
        py::arg("expert_width") = 0, py::arg("n_experts") = 0, py::arg("shared_scale") = 1.0,
        py::arg("stats") = py::none(), py::arg("bn") = 0);
  m.def("gemm_choose_bn", &gemm_choose_bn);
  m.def("gemm_grouped", &gemm_grouped, "grouped tcgen05 GEMM", py::arg("A"), py::arg("a_mn"),
        py::arg("B"), py::arg("b_mn"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi"),
        py::arg("out") = py::none(), py::arg("gu") = py::none(), py::arg("act") = py::none(),
        py::arg("row_scale") = py::none(), py::arg("expert_width") = 0, py::arg("mode") = 1,
        py::arg("tile_group") = py::none(), py::arg("k_start") = py::none(),
        py::arg("groups") = 1, py::arg("b_stride") = 0, py::arg("c_stride") = 0,
        py::arg("alpha") = 1.0);
  m.def("moe_plan", &moe_plan);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine, py::arg("src"), py::arg("token_pos"), py::arg("k"),
        py::arg("scale") = 1.0, py::arg("base") = py::none());
  m.def("flash_attn_fwd", &flash_attn_fwd);
  m.def("flash_attn_bwd", &flash_attn_bwd);
  m.def("dp_reduce_shard", &dp_reduce_shard, py::arg("grad"), py::arg("param"), py::arg("pad"),
        py::arg("slots"), py::arg("rank"), py::arg("lo"), py::arg("n"), py::arg("gs"),
        py::arg("sumsq_local"), py::arg("ticket"), py::arg("epoch"), py::arg("publish"),
        py::arg("epoch_dev") = py::none());
  m.def("dp_adamw_shard", &dp_adamw_shard, py::arg("grad"), py::arg("param"), py::arg("pad"),
        py::arg("slots"), py::arg("rank"), py::arg("lo"), py::arg("n"), py::arg("master"),
        py::arg("m"), py::arg("v"), py::arg("gs"), py::arg("lr"), py::arg("b1"), py::arg("b2"),
        py::arg("eps"), py::arg("wd"), py::arg("bc1"), py::arg("bc2"), py::arg("max_norm"),
        py::arg("norm_out"), py::arg("ticket"), py::arg("epoch"),
        py::arg("epoch_dev") = py::none(), py::arg("hyper") = py::none());
  m.def("dp_epoch_bump", [](torch::Tensor& e) {
    TORCH_CHECK(e.is_cuda() && e.scalar_type() == torch::kInt32, "epoch counter: int32 CUDA");
    const c10::cuda::CUDAGuard guard(e.device());
    raise_rc(cfb::fused_epoch_bump(e.data_ptr<int>(), at::cuda::getCurrentCUDAStream()),
             "dp_epoch_bump");
  });
  register_elementwise(m);
}
