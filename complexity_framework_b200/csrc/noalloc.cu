// Allocation-free weight-gradient GEMM (declared in noalloc.h).
//
// Same computation as the weight-gradient path of the framework's linear
// layers (split-K tcgen05 GEMM accumulating fp32 partial products with
// atomics, then a cast to bf16), except that the fp32 accumulator is the
// file-scope device array below instead of memory the caller allocates.
#include <cuda_bf16.h>

#include <mutex>

#include "gemm_tc.h"
#include "noalloc.h"

namespace {

// The accumulator and a private device error word.  In host code these names
// are host-side stand-ins, never device addresses: their device addresses come
// from cudaGetSymbolAddress (per device) below.
static __device__ __align__(256) float g_wgrad_acc[CFB_NOALLOC_MAX_ELEMS];
static __device__ __align__(256) int g_wgrad_err[4];

constexpr int kMaxDevices = 64;
struct DeviceSlots {
  float* acc = nullptr;
  int* err = nullptr;
  int num_sms = 0;
};
DeviceSlots g_slots[kMaxDevices];
std::mutex g_slots_mu;

// Looks up (once per device, with that device current) the device addresses
// of the accumulator and error word.
int resolve_slots(int dev, DeviceSlots* out) {
  std::lock_guard<std::mutex> lk(g_slots_mu);
  DeviceSlots& s = g_slots[dev];
  if (s.acc == nullptr) {
    void* acc = nullptr;
    void* err = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&acc, g_wgrad_acc);
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaGetSymbolAddress(&err, g_wgrad_err);
    if (e != cudaSuccess) return static_cast<int>(e);
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    s.acc = static_cast<float*>(acc);
    s.err = static_cast<int*>(err);
    s.num_sms = sms;
  }
  *out = s;
  return 0;
}

__global__ void cast_f32_to_bf16(const float* __restrict__ in, __nv_bfloat16* __restrict__ out,
                                 int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16(in[i]);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int cfb_weight_grad_noalloc(
    const void* dy, const void* x, int T, int N, int K, void* dw, cudaStream_t stream) {
  // report (and leave in place) an error that earlier work left pending, so
  // that this call never returns, or clears, a failure that is not its own
  const cudaError_t pending = cudaPeekAtLastError();
  if (pending != cudaSuccess) return static_cast<int>(pending);
  if (T <= 0 || N <= 0 || K <= 0) return -2;
  if (static_cast<uint64_t>(N) * static_cast<uint64_t>(K) > CFB_NOALLOC_MAX_ELEMS) return -1;
  // TMA operands: 16-byte aligned rows (N and K multiples of 8); epilogue: K % 32
  if (N % 8 != 0 || K % 32 != 0 || !aligned16(dy) || !aligned16(x) || !aligned16(dw)) return -2;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return -2;
  DeviceSlots slots;
  const int rc0 = resolve_slots(dev, &slots);
  if (rc0 != 0) return rc0;
  const size_t elems = static_cast<size_t>(N) * static_cast<size_t>(K);
  // the accumulator keeps the previous call's sums: clear what this call uses
  e = cudaMemsetAsync(slots.acc, 0, elems * sizeof(float), stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  cfb::GemmArgs g;
  g.A = dy;        // A(m = n_out, k = t) = dY[t, n_out]  (MN-major)
  g.lda = N;
  g.a_mn = true;
  g.B = x;         // B(n = k_in, k = t) = X[t, k_in]     (MN-major)
  g.ldb = K;
  g.b_mn = true;
  g.M = N;
  g.N = K;
  g.K = T;
  g.epi = cfb::EPI_F32_ATOMIC;
  g.num_sms = slots.num_sms;
  cfb::GemmEpi ep;
  ep.c = slots.acc;
  ep.ldc = K;
  ep.alpha = 1.0f;
  const int rc = cfb::gemm_tc_launch(g, ep, stream, slots.err);
  if (rc >= 1000) return rc;              // tensor-map encode failure: 1000 + CUresult
  if (rc < 0) return -3;                  // internal launch failure
  if (rc != 0) return rc;                 // cudaError_t
  const int grid = static_cast<int>((elems + 255) / 256 < 4096 ? (elems + 255) / 256 : 4096);
  cast_f32_to_bf16<<<grid, 256, 0, stream>>>(slots.acc, static_cast<__nv_bfloat16*>(dw),
                                             static_cast<int64_t>(elems));
  return static_cast<int>(cudaGetLastError());
}

extern "C" __attribute__((visibility("default"))) int cfb_weight_grad_noalloc_status(
    int out[4], cudaStream_t stream) {
  if (out == nullptr) return -2;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return -2;
  DeviceSlots slots;
  const int rc0 = resolve_slots(dev, &slots);
  if (rc0 != 0) return rc0;
  e = cudaMemcpyAsync(out, slots.err, 4 * sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemsetAsync(slots.err, 0, 4 * sizeof(int), stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaStreamSynchronize(stream));
}
