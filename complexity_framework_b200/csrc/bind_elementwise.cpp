// Python bindings of the memory-bound kernels (elementwise.cu).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <unordered_map>
#include <utility>

#include "kernels.h"

namespace py = pybind11;

namespace {

using cfb::bf16;

void chk(const torch::Tensor& t, torch::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be CUDA");
  TORCH_CHECK(t.scalar_type() == dt, name, " has wrong dtype ", t.scalar_type());
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
template <typename T>
T* P(const torch::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <typename T>
T* Popt(const c10::optional<torch::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
cudaStream_t cur() { return at::cuda::getCurrentCUDAStream(); }

// Accumulator slots for norm-weight gradients written straight to bf16: each
// slot is 1024 floats plus a ticket word, zero between launches (the last
// block of each launch re-zeroes its slot).  Calls take slots round-robin,
// so launches that share a slot are kSlots calls apart; launches that run
// concurrently on different streams must be fewer than kSlots calls apart.
constexpr int kSlotFloats = 1024, kSlotStride = 1024 + 32, kSlots = 256;
std::mutex g_slot_mu;
std::unordered_map<int, std::pair<torch::Tensor, int>> g_slots;

std::pair<float*, int*> grad_slot(int device, int64_t n) {
  TORCH_CHECK(n <= kSlotFloats, "norm-weight gradient slot holds at most ", kSlotFloats,
              " floats");
  std::lock_guard<std::mutex> lk(g_slot_mu);
  auto it = g_slots.find(device);
  if (it == g_slots.end()) {
    auto t = torch::zeros({int64_t(kSlots) * kSlotStride},
                          torch::dtype(torch::kFloat32).device(torch::kCUDA, device));
    it = g_slots.emplace(device, std::make_pair(t, 0)).first;
  }
  const int i = it->second.second;
  it->second.second = (i + 1) % kSlots;
  float* base = it->second.first.data_ptr<float>() + int64_t(i) * kSlotStride;
  return {base, reinterpret_cast<int*>(base + kSlotFloats)};
}

void rmsnorm_fwd(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& y,
                 torch::Tensor& rstd, double eps) {
  chk(x, torch::kBFloat16, "x");
  chk(w, torch::kBFloat16, "w");
  chk(y, torch::kBFloat16, "y");
  chk(rstd, torch::kFloat32, "rstd");
  const int64_t H = x.size(-1);
  TORCH_CHECK(H % 8 == 0 && w.numel() == H, "rmsnorm: H must be a multiple of 8");
  const int64_t T = x.numel() / H;
  TORCH_CHECK(y.numel() == x.numel() && rstd.numel() >= T, "rmsnorm: output sizes");
  const c10::cuda::CUDAGuard g(x.device());
  cfb::rmsnorm_fwd(P<bf16>(x), P<bf16>(w), P<bf16>(y), P<float>(rstd), T, static_cast<int>(H),
                   static_cast<float>(eps), cur());
}

void rmsnorm_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& w,
                 const torch::Tensor& rstd, const c10::optional<torch::Tensor>& dres,
                 torch::Tensor& dx, torch::Tensor& dw) {
  chk(dy, torch::kBFloat16, "dy");
  chk(x, torch::kBFloat16, "x");
  chk(w, torch::kBFloat16, "w");
  chk(rstd, torch::kFloat32, "rstd");
  chk(dx, torch::kBFloat16, "dx");
  const bool bf16_dw = dw.scalar_type() == torch::kBFloat16;
  chk(dw, bf16_dw ? torch::kBFloat16 : torch::kFloat32, "dw");
  if (dres.has_value()) chk(*dres, torch::kBFloat16, "dres");
  const int64_t H = x.size(-1);
  TORCH_CHECK(H % 8 == 0, "rmsnorm: H must be a multiple of 8");
  const int64_t T = x.numel() / H;
  TORCH_CHECK(dy.numel() == x.numel() && dx.numel() == x.numel() && dw.numel() == H,
              "rmsnorm_bwd sizes");
  TORCH_CHECK(!bf16_dw || (H <= 1024 && T < (int64_t(1) << 31)),
              "rmsnorm_bwd: a bf16 dw needs H <= 1024 (pass an fp32 accumulator otherwise)");
  const c10::cuda::CUDAGuard g(x.device());
  if (bf16_dw) {
    auto slot = grad_slot(x.get_device(), H);
    cfb::rmsnorm_bwd(P<bf16>(dy), P<bf16>(x), P<bf16>(w), P<float>(rstd), Popt<bf16>(dres),
                     P<bf16>(dx), slot.first, T, static_cast<int>(H), P<bf16>(dw), slot.second,
                     cur());
  } else {
    cfb::rmsnorm_bwd(P<bf16>(dy), P<bf16>(x), P<bf16>(w), P<float>(rstd), Popt<bf16>(dres),
                     P<bf16>(dx), P<float>(dw), T, static_cast<int>(H), nullptr, nullptr, cur());
  }
}

void qk_norm_rope_fwd(const torch::Tensor& kqv, const torch::Tensor& qw, const torch::Tensor& kw,
                      const torch::Tensor& cos_t, const torch::Tensor& sin_t,
                      const c10::optional<torch::Tensor>& pos, torch::Tensor& q, torch::Tensor& k,
                      torch::Tensor& v, torch::Tensor& rstd, int64_t B, int64_t S, int64_t Hq,
                      int64_t Hkv, int64_t D, double eps, bool qk_norm, bool q_tm) {
  TORCH_CHECK(B * S * (Hq + 2 * Hkv) < (int64_t(1) << 31), "qk_norm_rope: too many (token, head) items");
  chk(kqv, torch::kBFloat16, "kqv");
  chk(qw, torch::kBFloat16, "q_norm.weight");
  chk(kw, torch::kBFloat16, "k_norm.weight");
  chk(cos_t, torch::kFloat32, "cos");
  chk(sin_t, torch::kFloat32, "sin");
  chk(q, torch::kBFloat16, "q");
  chk(k, torch::kBFloat16, "k");
  chk(v, torch::kBFloat16, "v");
  chk(rstd, torch::kFloat32, "rstd");
  TORCH_CHECK(D == 64 || D == 128, "qk_norm_rope: head_dim must be 64 or 128");
  TORCH_CHECK(kqv.numel() == B * S * (Hq + 2 * Hkv) * D, "kqv size");
  TORCH_CHECK(q.numel() == B * Hq * S * D && k.numel() == B * Hkv * S * D &&
                  v.numel() == B * Hkv * S * D,
              "q/k/v size");
  TORCH_CHECK(rstd.numel() >= B * S * (Hq + Hkv), "rstd size");
  TORCH_CHECK(cos_t.size(-1) == D / 2, "cos table must be [P, D/2]");
  if (pos.has_value()) {
    chk(*pos, torch::kInt32, "pos");
  } else {
    TORCH_CHECK(cos_t.size(0) >= S, "cos table shorter than sequence");
  }
  const c10::cuda::CUDAGuard g(kqv.device());
  cfb::qk_norm_rope_fwd(P<bf16>(kqv), P<bf16>(qw), P<bf16>(kw), P<float>(cos_t), P<float>(sin_t),
                        Popt<int32_t>(pos), P<bf16>(q), P<bf16>(k), P<bf16>(v), P<float>(rstd),
                        static_cast<int>(B), static_cast<int>(S), static_cast<int>(Hq),
                        static_cast<int>(Hkv), static_cast<int>(D), static_cast<float>(eps),
                        qk_norm, q_tm, cur());
}

void qk_norm_rope_bwd(const torch::Tensor& dq, const torch::Tensor& dk, const torch::Tensor& dv,
                      const torch::Tensor& kqv, const torch::Tensor& qw, const torch::Tensor& kw,
                      const torch::Tensor& cos_t, const torch::Tensor& sin_t,
                      const c10::optional<torch::Tensor>& pos, const torch::Tensor& rstd,
                      torch::Tensor& dkqv, torch::Tensor& dqw, torch::Tensor& dkw, int64_t B,
                      int64_t S, int64_t Hq, int64_t Hkv, int64_t D, bool qk_norm, bool q_tm) {
  TORCH_CHECK(B * S * (Hq + 2 * Hkv) < (int64_t(1) << 31), "qk_norm_rope: too many (token, head) items");
  chk(dq, torch::kBFloat16, "dq");
  chk(dk, torch::kBFloat16, "dk");
  chk(dv, torch::kBFloat16, "dv");
  chk(kqv, torch::kBFloat16, "kqv");
  chk(dkqv, torch::kBFloat16, "dkqv");
  const bool bf16_dw = dqw.scalar_type() == torch::kBFloat16;
  chk(dqw, bf16_dw ? torch::kBFloat16 : torch::kFloat32, "dqw");
  chk(dkw, bf16_dw ? torch::kBFloat16 : torch::kFloat32, "dkw");
  TORCH_CHECK(dqw.numel() == D && dkw.numel() == D, "dqw/dkw size");
  chk(rstd, torch::kFloat32, "rstd");
  TORCH_CHECK(D == 64 || D == 128, "qk_norm_rope: head_dim must be 64 or 128");
  TORCH_CHECK(dkqv.numel() == kqv.numel() && kqv.numel() == B * S * (Hq + 2 * Hkv) * D,
              "dkqv size");
  if (pos.has_value()) chk(*pos, torch::kInt32, "pos");
  const c10::cuda::CUDAGuard g(kqv.device());
  float* aq = nullptr;
  float* ak = nullptr;
  int* ticket = nullptr;
  if (bf16_dw) {
    auto slot = grad_slot(kqv.get_device(), 2 * D);
    aq = slot.first;
    ak = slot.first + D;
    ticket = slot.second;
  } else {
    aq = P<float>(dqw);
    ak = P<float>(dkw);
  }
  cfb::qk_norm_rope_bwd(P<bf16>(dq), P<bf16>(dk), P<bf16>(dv), P<bf16>(kqv), P<bf16>(qw),
                        P<bf16>(kw), P<float>(cos_t), P<float>(sin_t), Popt<int32_t>(pos),
                        P<float>(rstd), P<bf16>(dkqv), aq, ak, static_cast<int>(B),
                        static_cast<int>(S), static_cast<int>(Hq), static_cast<int>(Hkv),
                        static_cast<int>(D), qk_norm, q_tm,
                        bf16_dw ? P<bf16>(dqw) : nullptr, bf16_dw ? P<bf16>(dkw) : nullptr,
                        ticket, cur());
}

void embedding_fwd(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out) {
  chk(ids, torch::kInt64, "ids");
  chk(table, torch::kBFloat16, "table");
  chk(out, torch::kBFloat16, "out");
  const int64_t H = table.size(1);
  TORCH_CHECK(H % 8 == 0 && out.numel() == ids.numel() * H, "embedding sizes");
  const c10::cuda::CUDAGuard g(ids.device());
  cfb::embedding_fwd(P<int64_t>(ids), P<bf16>(table), P<bf16>(out), ids.numel(),
                     static_cast<int>(H), table.size(0), cur());
}

void embedding_bwd_sorted(const torch::Tensor& sorted_ids, const torch::Tensor& order,
                          const torch::Tensor& dy, torch::Tensor& dtable) {
  chk(sorted_ids, torch::kInt64, "sorted_ids");
  chk(order, torch::kInt64, "order");
  chk(dy, torch::kBFloat16, "dy");
  chk(dtable, torch::kFloat32, "dtable");
  const int64_t H = dtable.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 1024, "embedding_bwd_sorted: H % 8 == 0 and H <= 1024");
  TORCH_CHECK(order.numel() == sorted_ids.numel() && dy.numel() == sorted_ids.numel() * H,
              "embedding_bwd_sorted sizes");
  const c10::cuda::CUDAGuard g(dy.device());
  cfb::embedding_bwd_sorted(P<int64_t>(sorted_ids), P<int64_t>(order), P<bf16>(dy),
                            P<float>(dtable), sorted_ids.numel(), static_cast<int>(H),
                            dtable.size(0), cur());
}

void embedding_bwd(const torch::Tensor& ids, const torch::Tensor& dy, torch::Tensor& dtable) {
  chk(ids, torch::kInt64, "ids");
  chk(dy, torch::kBFloat16, "dy");
  chk(dtable, torch::kFloat32, "dtable");
  const int64_t H = dtable.size(1);
  TORCH_CHECK(H % 8 == 0 && dy.numel() == ids.numel() * H, "embedding_bwd sizes");
  const c10::cuda::CUDAGuard g(ids.device());
  cfb::embedding_bwd(P<int64_t>(ids), P<bf16>(dy), P<float>(dtable), ids.numel(),
                     static_cast<int>(H), dtable.size(0), cur());
}

void ce_loss_grad(torch::Tensor& logits, const torch::Tensor& stats, int64_t ntiles,
                  const torch::Tensor& targets, torch::Tensor& loss, const torch::Tensor& scale,
                  int64_t ignore_index) {
  chk(logits, torch::kBFloat16, "logits");
  chk(stats, torch::kFloat32, "stats");
  chk(targets, torch::kInt64, "targets");
  chk(loss, torch::kFloat32, "loss");
  chk(scale, torch::kFloat32, "scale");
  TORCH_CHECK(logits.dim() == 2 && logits.size(1) % 8 == 0, "logits must be [T, V], V % 8 == 0");
  const int64_t T = logits.size(0);
  TORCH_CHECK(targets.numel() == T && loss.numel() == T && stats.numel() >= T * ntiles * 2,
              "ce sizes");
  const c10::cuda::CUDAGuard g(logits.device());
  cfb::ce_loss_grad(P<bf16>(logits), P<float>(stats), static_cast<int>(ntiles),
                    P<int64_t>(targets), P<float>(loss), P<float>(scale), T,
                    static_cast<int>(logits.size(1)), ignore_index, cur());
}

void route_scales(const torch::Tensor& ids, const torch::Tensor& table, const torch::Tensor& rw,
                  torch::Tensor& out, int64_t E, double routed_scale) {
  chk(ids, torch::kInt64, "ids");
  chk(table, torch::kInt64, "route_table");
  chk(rw, torch::kFloat32, "route_weights");
  chk(out, torch::kFloat32, "out");
  TORCH_CHECK(E >= 1 && E <= 16, "route_scales supports up to 16 experts");
  TORCH_CHECK(table.dim() == 2 && rw.numel() == table.size(0), "route table/weights");
  TORCH_CHECK(out.numel() == ids.numel() * E, "route_scales out size");
  const c10::cuda::CUDAGuard g(ids.device());
  cfb::route_scales(P<int64_t>(ids), P<int64_t>(table), P<float>(rw), P<float>(out), ids.numel(),
                    static_cast<int>(table.size(0)), table.size(1), static_cast<int>(E),
                    static_cast<float>(routed_scale), cur());
}

void adamw_flat(torch::Tensor& p, torch::Tensor& m, torch::Tensor& v, const torch::Tensor& g,
                const c10::optional<torch::Tensor>& p_out, double lr, double b1, double b2,
                double eps, double wd, double bc1, double bc2,
                const c10::optional<torch::Tensor>& clip,
                const c10::optional<torch::Tensor>& hyper) {
  chk(p, torch::kFloat32, "p");
  chk(m, torch::kFloat32, "exp_avg");
  chk(v, torch::kFloat32, "exp_avg_sq");
  chk(g, torch::kBFloat16, "grad");
  const int64_t n = p.numel();
  TORCH_CHECK(m.numel() == n && v.numel() == n && g.numel() == n, "adamw sizes");
  if (p_out.has_value()) {
    chk(*p_out, torch::kBFloat16, "p_out");
    TORCH_CHECK(p_out->numel() == n, "p_out size");
  }
  if (clip.has_value()) chk(*clip, torch::kFloat32, "clip");
  if (hyper.has_value()) {
    chk(*hyper, torch::kFloat32, "hyper");
    TORCH_CHECK(hyper->numel() >= 3, "hyper holds (lr, bias correction 1, bias correction 2)");
  }
  const c10::cuda::CUDAGuard guard(p.device());
  cfb::adamw_flat(P<float>(p), P<float>(m), P<float>(v), P<bf16>(g), Popt<bf16>(p_out), n,
                  static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2),
                  static_cast<float>(eps), static_cast<float>(wd), static_cast<float>(bc1),
                  static_cast<float>(bc2), Popt<float>(clip), Popt<float>(hyper), cur());
}

void sumsq_bf16(const torch::Tensor& g, torch::Tensor& out) {
  chk(g, torch::kBFloat16, "g");
  chk(out, torch::kFloat32, "out");
  const c10::cuda::CUDAGuard guard(g.device());
  cfb::sumsq_bf16(P<bf16>(g), g.numel(), P<float>(out), cur());
}

void clip_coef(const torch::Tensor& sumsq, double max_norm, torch::Tensor& clip,
               torch::Tensor& norm) {
  const c10::cuda::CUDAGuard guard(sumsq.device());
  cfb::clip_coef(P<float>(sumsq), static_cast<float>(max_norm), P<float>(clip), P<float>(norm),
                 cur());
}

void paged_attention(const torch::Tensor& q, const torch::Tensor& k_pool,
                     const torch::Tensor& v_pool, const torch::Tensor& page_table,
                     const torch::Tensor& cu_q, const torch::Tensor& kv_lens, torch::Tensor& out,
                     double scale, int64_t max_q_len, int64_t pages_per_split) {
  chk(q, torch::kBFloat16, "q");
  chk(k_pool, torch::kBFloat16, "k_pool");
  chk(v_pool, torch::kBFloat16, "v_pool");
  chk(page_table, torch::kInt32, "page_table");
  chk(cu_q, torch::kInt32, "cu_q");
  chk(kv_lens, torch::kInt32, "kv_lens");
  chk(out, torch::kBFloat16, "out");
  TORCH_CHECK(q.dim() == 3 && k_pool.dim() == 4 && v_pool.sizes() == k_pool.sizes(),
              "q [N,Hq,D], pools [pages,page,Hkv,D]");
  const int64_t N = q.size(0), Hq = q.size(1), D = q.size(2);
  const int64_t page = k_pool.size(1), Hkv = k_pool.size(2);
  TORCH_CHECK(k_pool.size(3) == D && Hq % Hkv == 0, "head shapes");
  const int64_t num_seqs = kv_lens.numel();
  TORCH_CHECK(cu_q.numel() == num_seqs + 1 && page_table.size(0) == num_seqs, "batch metadata");
  TORCH_CHECK(out.sizes() == q.sizes(), "out shape");
  (void)max_q_len;
  const c10::cuda::CUDAGuard g(q.device());
  const int max_pages = static_cast<int>(page_table.size(1));
  int pps = 0, splits = 0;
  cfb::paged_attention_split(static_cast<int>(N), static_cast<int>(Hkv),
                             max_pages * static_cast<int>(page),
                             at::cuda::getCurrentDeviceProperties()->multiProcessorCount, &pps,
                             &splits);
  if (pages_per_split > 0) {  // caller's split (tuning); 0 keeps the automatic choice
    pps = static_cast<int>(pages_per_split);
    splits = (max_pages + pps - 1) / pps;
  }
  torch::Tensor ws_o, ws_lse;
  if (splits > 1) {
    const auto f32 = q.options().dtype(torch::kFloat32);
    ws_o = torch::empty({N * Hq * splits * D}, f32);
    ws_lse = torch::empty({N * Hq * splits}, f32);
  }
  const int rc = cfb::paged_attention(
      P<bf16>(q), P<bf16>(k_pool), P<bf16>(v_pool), P<int32_t>(page_table), P<int32_t>(cu_q),
      P<int32_t>(kv_lens), P<bf16>(out), splits > 1 ? ws_o.data_ptr<float>() : nullptr,
      splits > 1 ? ws_lse.data_ptr<float>() : nullptr, static_cast<int>(N),
      static_cast<int>(num_seqs), max_pages, static_cast<int>(Hq), static_cast<int>(Hkv),
      static_cast<int>(D), static_cast<int>(page), pps, splits, static_cast<float>(scale), cur());
  TORCH_CHECK(rc == 0, "paged_attention failed with code ", rc);
}

void paged_qkv_rope(const torch::Tensor& kqv, const c10::optional<torch::Tensor>& qw,
                    const c10::optional<torch::Tensor>& kw, const torch::Tensor& cos_t,
                    const torch::Tensor& sin_t, const torch::Tensor& pos,
                    const torch::Tensor& slots, torch::Tensor& q_out, torch::Tensor& k_layer,
                    torch::Tensor& v_layer, double eps) {
  chk(kqv, torch::kBFloat16, "kqv");
  chk(q_out, torch::kBFloat16, "q_out");
  chk(k_layer, torch::kBFloat16, "k_layer");
  chk(v_layer, torch::kBFloat16, "v_layer");
  chk(cos_t, torch::kFloat32, "cos");
  chk(sin_t, torch::kFloat32, "sin");
  chk(pos, torch::kLong, "positions");
  chk(slots, torch::kLong, "slots");
  TORCH_CHECK(q_out.dim() == 3 && k_layer.dim() == 4 && v_layer.sizes() == k_layer.sizes(),
              "q_out [N,Hq,D], pools [pages,page,Hkv,D]");
  const int64_t N = q_out.size(0), Hq = q_out.size(1), D = q_out.size(2);
  const int64_t Hkv = k_layer.size(2);
  TORCH_CHECK(k_layer.size(3) == D && (D == 64 || D == 128), "head dim 64 or 128");
  TORCH_CHECK(kqv.dim() == 2 && kqv.size(0) == N && kqv.size(1) == (Hq + 2 * Hkv) * D,
              "kqv [N, (2 Hkv + Hq) D]");
  TORCH_CHECK(pos.numel() == N && slots.numel() == N, "one position and slot per token");
  TORCH_CHECK(cos_t.dim() == 2 && cos_t.size(1) == D / 2 && sin_t.sizes() == cos_t.sizes(),
              "cos/sin tables [P, D/2]");
  const bool norm = qw.has_value();
  TORCH_CHECK(norm == kw.has_value(), "q and k norm weights go together");
  if (norm) {
    chk(*qw, torch::kBFloat16, "q_norm weight");
    chk(*kw, torch::kBFloat16, "k_norm weight");
    TORCH_CHECK(qw->numel() == D && kw->numel() == D, "norm weights [D]");
  }
  const c10::cuda::CUDAGuard g(kqv.device());
  const int rc = cfb::paged_qkv_rope(
      P<bf16>(kqv), norm ? P<bf16>(*qw) : nullptr, norm ? P<bf16>(*kw) : nullptr,
      P<float>(cos_t), P<float>(sin_t), P<int64_t>(pos), P<int64_t>(slots), P<bf16>(q_out),
      P<bf16>(k_layer), P<bf16>(v_layer), static_cast<int>(N), static_cast<int>(Hq),
      static_cast<int>(Hkv), static_cast<int>(D), static_cast<float>(eps), norm, cur());
  TORCH_CHECK(rc == 0, "paged_qkv_rope failed with code ", rc);
}

void skinny_finish(const torch::Tensor& acc, const c10::optional<torch::Tensor>& resid,
                   torch::Tensor& out, double alpha) {
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == torch::kFloat32 && acc.dim() == 2 &&
                  acc.stride(1) == 1, "acc: fp32 [N, >=M] row-major");
  chk(out, torch::kBFloat16, "out");
  TORCH_CHECK(out.dim() == 2, "out [M, N]");
  const int64_t M = out.size(0), N = out.size(1);
  TORCH_CHECK(acc.size(0) == N && acc.size(1) >= M, "acc [N, >=M]");
  if (resid.has_value()) {
    chk(*resid, torch::kBFloat16, "residual");
    TORCH_CHECK(resid->numel() == M * N, "residual [M, N]");
  }
  const c10::cuda::CUDAGuard g(out.device());
  cfb::skinny_finish(P<float>(acc), static_cast<int>(acc.stride(0)),
                     resid.has_value() ? P<bf16>(*resid) : nullptr, P<bf16>(out),
                     static_cast<int>(M), static_cast<int>(N), static_cast<float>(alpha), cur());
}

void skinny_swiglu(const torch::Tensor& acc, const torch::Tensor& row_scale, torch::Tensor& act,
                   int64_t shared_width, int64_t expert_width, int64_t n_experts,
                   double shared_scale) {
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == torch::kFloat32 && acc.dim() == 2 &&
                  acc.stride(1) == 1, "acc: fp32 [2A, >=T] row-major");
  chk(act, torch::kBFloat16, "act");
  chk(row_scale, torch::kFloat32, "row_scale");
  TORCH_CHECK(act.dim() == 2, "act [T, A]");
  const int64_t T = act.size(0), A = act.size(1);
  TORCH_CHECK(A % 128 == 0 && acc.size(0) == 2 * A && acc.size(1) >= T, "acc [2A, >=T]");
  TORCH_CHECK(A == shared_width || (expert_width > 0 && n_experts > 0 &&
                                    row_scale.numel() >= T * n_experts),
              "row_scale [T, n_experts]");
  const c10::cuda::CUDAGuard g(act.device());
  cfb::skinny_swiglu(P<float>(acc), static_cast<int>(acc.stride(0)), P<float>(row_scale),
                     P<bf16>(act), static_cast<int>(T), static_cast<int>(A),
                     static_cast<int>(shared_width), static_cast<int>(expert_width > 0 ? expert_width : 1),
                     static_cast<int>(n_experts), static_cast<float>(shared_scale), cur());
}

// geom: 10 ints per job (rows, cols, s_div, s_hi, s_lo, s_cs, d_div, d_hi, d_lo,
// d_cs), element offsets relative to each tensor's data pointer.  Every job's
// largest source and destination offsets are checked against the tensors.
void copy_jobs(const std::vector<torch::Tensor>& srcs, const std::vector<torch::Tensor>& dsts,
               const std::vector<int64_t>& geom) {
  const size_t n = srcs.size();
  TORCH_CHECK(n >= 1 && n <= static_cast<size_t>(cfb::kMaxCopyJobs) && dsts.size() == n &&
                  geom.size() == 10 * n,
              "copy_jobs: 1..", cfb::kMaxCopyJobs, " jobs with 10 geometry values each");
  cfb::CopyJobs jobs;
  jobs.n = static_cast<int>(n);
  auto max_off = [](int64_t rows, int64_t cols, int64_t div, int64_t hi, int64_t lo,
                    int64_t cs) {
    const int64_t r = rows - 1;
    const int64_t inner = r < div - 1 ? r : div - 1;
    return (r / div) * hi + inner * lo + (cols - 1) * cs;
  };
  for (size_t i = 0; i < n; ++i) {
    const int64_t* g = geom.data() + 10 * i;
    const torch::Tensor& s = srcs[i];
    const torch::Tensor& d = dsts[i];
    TORCH_CHECK(s.is_cuda() && d.is_cuda() && s.get_device() == d.get_device(),
                "copy_jobs: CUDA tensors on one device");
    TORCH_CHECK(s.scalar_type() == torch::kFloat32 || s.scalar_type() == torch::kBFloat16,
                "copy_jobs: source must be fp32 or bf16");
    TORCH_CHECK(d.scalar_type() == torch::kBFloat16, "copy_jobs: destination must be bf16");
    TORCH_CHECK(g[0] > 0 && g[1] > 0 && g[0] < (1 << 30) && g[1] < (1 << 30) && g[2] > 0 &&
                    g[6] > 0 && g[3] >= 0 && g[4] >= 0 && g[5] >= 0 && g[7] >= 0 &&
                    g[8] >= 0 && g[9] >= 0,
                "copy_jobs: bad geometry");
    TORCH_CHECK(max_off(g[0], g[1], g[2], g[3], g[4], g[5]) < s.numel(),
                "copy_jobs: job ", i, " reads past its source");
    TORCH_CHECK(max_off(g[0], g[1], g[6], g[7], g[8], g[9]) < d.numel(),
                "copy_jobs: job ", i, " writes past its destination");
    cfb::CopyJob& J = jobs.j[i];
    J.src = s.data_ptr();
    J.dst = P<bf16>(d);
    J.src_f32 = s.scalar_type() == torch::kFloat32;
    J.rows = static_cast<int>(g[0]);
    J.cols = static_cast<int>(g[1]);
    J.s_div = static_cast<int>(std::min<int64_t>(g[2], 1 << 30));
    J.s_hi = g[3];
    J.s_lo = g[4];
    J.s_cs = g[5];
    J.d_div = static_cast<int>(std::min<int64_t>(g[6], 1 << 30));
    J.d_hi = g[7];
    J.d_lo = g[8];
    J.d_cs = g[9];
  }
  const c10::cuda::CUDAGuard guard(srcs[0].device());
  cfb::copy_jobs(jobs, cur());
}

}  // namespace

void register_elementwise(pybind11::module& m) {
  m.def("copy_jobs", &copy_jobs);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("embedding_bwd_sorted", &embedding_bwd_sorted);
  m.def("ce_loss_grad", &ce_loss_grad);
  m.def("route_scales", &route_scales);
  m.def("adamw_flat", &adamw_flat, py::arg("p"), py::arg("m"), py::arg("v"), py::arg("g"),
        py::arg("p_out"), py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"),
        py::arg("wd"), py::arg("bc1"), py::arg("bc2"), py::arg("clip"),
        py::arg("hyper") = py::none());
  m.def("sumsq_bf16", &sumsq_bf16);
  m.def("clip_coef", &clip_coef);
  m.def("paged_attention", &paged_attention, py::arg("q"), py::arg("k_pool"), py::arg("v_pool"),
        py::arg("page_table"), py::arg("cu_q"), py::arg("kv_lens"), py::arg("out"),
        py::arg("scale"), py::arg("max_q_len"), py::arg("pages_per_split") = 0);
  m.def("paged_qkv_rope", &paged_qkv_rope);
  m.def("skinny_finish", &skinny_finish);
  m.def("skinny_swiglu", &skinny_swiglu);
}
