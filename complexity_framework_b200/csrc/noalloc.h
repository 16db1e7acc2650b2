// Allocation-free weight-gradient entry point.
//
// This entry point has no counterpart in the reference framework.  It exists
// for callers that cannot allocate device memory while they run: code executing
// inside another runtime's memory budget (plugins of inference engines or
// serving frameworks that forbid cudaMalloc after initialisation), real-time
// loops that must never block on the driver's allocator, and C/C++ hosts that
// link this library without PyTorch's caching allocator.  They pass their own
// inputs and output; the fp32 accumulation buffer the split-K GEMM needs is a
// fixed-size array inside this library instead of a per-call allocation.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

// Largest output (N * K fp32 elements) the built-in accumulator holds:
// 4 Mi floats = 16 MiB of device memory, reserved on every GPU that loads the
// library until the process exits.
#define CFB_NOALLOC_MAX_ELEMS (4u * 1024u * 1024u)

#ifdef __cplusplus
extern "C" {
#endif

// dW[N, K] (bf16, row-major) = dY^T X for dY [T, N] and X [T, K] (bf16, row-major,
// leading dimensions N and K), i.e. the weight gradient of y = x W^T.
// Allocates nothing.  Return codes:
//    0          the work was enqueued on `stream`
//   -1          N*K exceeds CFB_NOALLOC_MAX_ELEMS
//   -2          bad shape, alignment or device index
//   -3          internal launch failure (the driver's tensor-map entry point is
//               missing, or the GEMM rejected its configuration)
//   1..999      a cudaError_t from this call's own CUDA calls, or an error that
//               earlier work on this thread left pending (returned unchanged
//               and left in place: this call then enqueues nothing)
//   1000+r      the driver refused to encode an operand tensor map (CUresult r)
// A device-side failure (a bounded wait inside the GEMM that timed out) is
// not visible in the return code: read it with cfb_weight_grad_noalloc_status.
//
// Use:
//  * The first call on a device looks up the device address of the built-in
//    accumulator for that device (cudaGetSymbolAddress, with that device
//    current); make that first call before any stream capture.
//  * All calls on a device share the one accumulator; it is cleared at the
//    start of every call, and its contents after a call are undefined.  Calls
//    whose executions overlap on the GPU (different streams without ordering)
//    race on it: order them on one stream or with events.
//  * `stream` may be 0 (the legacy default stream).
int cfb_weight_grad_noalloc(const void* dy, const void* x, int T, int N, int K, void* dw,
                            cudaStream_t stream);

// Device-side status of the calls on the current device: waits for `stream`,
// copies the error word into out[4] (out[0]: first error code, 0 = none;
// 1: bounded wait of a stage that never filled, 2: of a stage that never
// emptied, 3: of the accumulator hand-off; out[1]: site; out[2]: block;
// out[3]: number of errors) and clears it.  Allocates nothing.  Returns 0, or
// a cudaError_t / -2 like cfb_weight_grad_noalloc.
int cfb_weight_grad_noalloc_status(int out[4], cudaStream_t stream);

#ifdef __cplusplus
}
#endif
