// Host interface of the tcgen05 GEMM (see gemm_tc.cu for the kernel design).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace cfb {

enum GemmEpilogue : int {
  EPI_STORE = 0,       // C(bf16) = alpha * acc
  EPI_RESID = 1,       // C(bf16) = alpha * acc + R(bf16)
  EPI_SWIGLU_FWD = 2,  // gate|up tile -> GU(bf16 pre-activations), ACT = silu(g)*u*scale
  EPI_SWIGLU_BWD = 3,  // acc = d(ACT) -> C = d(GU) using saved GU
  EPI_F32 = 4,         // C(fp32) = alpha * acc
  EPI_F32_ACC = 5,     // C(fp32) += alpha * acc
  EPI_F32_ATOMIC = 7,  // C(fp32) += alpha * acc with atomics; K may be split across CTAs
  EPI_CE_STATS = 6,    // C(bf16) logits = alpha*acc; stats[row, N/128] = (max, sumexp); BN=256
  EPI_PEER_STORE = 8,  // reduce-scatter partials: owner = row / peer_rows; fp32 tile stored
                       // over NVLink into peer_c[owner][sync.rank][row % peer_rows][col]
};

constexpr int kMaxSeg = 8;

// Device barrier over symmetric-memory signal pads (int[rounds][kMaxSeg] per
// rank).  `role` 1: the TMA producer waits before its first load (operands
// that live in peer memory must be written); role 2: the epilogue waits
// before its first peer store (peer destinations must be cleared).  With
// `signal`, CTA 0 first announces this rank's arrival.  world == 0: none.
struct DistSync {
  int* pad[kMaxSeg] = {};
  int world = 0;
  int rank = 0;
  int round = 0;
  int epoch = 0;
  int role = 0;
  int signal = 0;
};

// Width (in activation columns) of one gate block in the packed gate|up weight:
// packed rows [256j, 256j+128) are gate rows [128j, 128j+128) and rows
// [256j+128, 256j+256) the matching up rows.
constexpr int kSwigluBlock = 128;

// All-gather of A's row shards performed inside the GEMM: warp 2 of every CTA
// copies 128-row chunks of the peers' shards (P2P loads) into this rank's
// gathered buffer `dst` (the A operand) and publishes a per-chunk flag; the
// TMA producer waits for a chunk's flag before loading its rows.  Tiles of
// this rank's own rows are scheduled first.  src[q] is rank q's gathered
// buffer, whose rows [q*rows, (q+1)*rows) hold q's shard.
struct AgCopy {
  const __nv_bfloat16* src[kMaxSeg] = {};
  __nv_bfloat16* dst = nullptr;
  int* flags = nullptr;  // one per 128-row chunk of dst
  int rows = 0;          // rows per rank
  int cols = 0;          // row length (elements) of src/dst
  int epoch = 0;
  int active = 0;
};

// Grouped GEMMs (expert-parallel work inside one launch).
//  mode 1, row-grouped: the A rows are sorted into per-group segments padded to
//    the 256-row tile; tile_group[m_tile] is the group of each 256-row tile (< 0:
//    no work) and B's storage rows of group g start at g * b_stride (N rows of a
//    K-major B, K rows of an MN-major B).
//  mode 2, K-grouped (weight gradients): group g multiplies the K rows
//    [k_start[g], k_start[g+1]) of MN-major A and B (multiples of 64) into output
//    rows [g * c_stride, g * c_stride + M); work units are (group, tile, K slice).
// The tables live in device memory, so segment sizes never reach the host.
struct GemmGroups {
  int mode = 0;
  const int* tile_group = nullptr;
  const int* k_start = nullptr;
  int ngroups = 0;
  int64_t b_stride = 0;
  int64_t c_stride = 0;
};

struct GemmEpi {
  void* c = nullptr;
  int64_t ldc = 0;
  const __nv_bfloat16* r = nullptr;
  int64_t ldr = 0;
  float alpha = 1.0f;
  __nv_bfloat16* gu = nullptr;
  int64_t ldgu = 0;
  __nv_bfloat16* act = nullptr;
  int64_t ldact = 0;
  const float* row_scale = nullptr;  // [M, n_experts]
  int shared_width = 0;
  int expert_width = 1;
  int n_experts = 0;
  float shared_scale = 1.0f;
  float* stats = nullptr;  // [M, 2*ceil(N/BN)] float2 (one per 128-column half tile)
  float* peer_c[kMaxSeg] = {};  // EPI_PEER_STORE: every rank's [world][peer_rows][ldc] fp32 slots
  int64_t peer_rows = 0;        // rows owned by each rank
  DistSync sync;
  AgCopy ag;
  GemmGroups grp;
};

struct GemmArgs {
  const void* A = nullptr;
  int64_t lda = 0;
  bool a_mn = false;
  const void* B = nullptr;
  int64_t ldb = 0;
  bool b_mn = false;
  int M = 0, N = 0, K = 0;
  int epi = EPI_STORE;
  int bn = 0;  // 0 = choose
  int num_sms = 148;
  // Operand segments (all-gather fused into the GEMM): when a_nseg > 0 the A
  // matrix is the concatenation, along its storage rows (M for K-major, K for
  // MN-major), of a_nseg matrices of a_seg_rows rows each, at A_seg[i] (peer
  // memory allowed; loads are plain TMA, never multicast).  Same for B.
  const void* A_seg[kMaxSeg] = {};
  int a_nseg = 0;
  int64_t a_seg_rows = 0;
  const void* B_seg[kMaxSeg] = {};
  int b_nseg = 0;
  int64_t b_seg_rows = 0;
};

int gemm_tc_launch(const GemmArgs& g, const GemmEpi& ep, cudaStream_t stream, int* err);
int choose_bn(int M, int N, int num_sms);
int make_tmap_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                 int box_inner, int box_outer);
// Tiled map of `rank` (<= 5) dims given innermost first; byte_strides[i] is the
// stride of dim i+1.  bf16 or fp32 elements, 128-byte swizzle or none.
int make_tmap_nd(CUtensorMap* map, const void* base, int rank, const int64_t* dims,
                 const int64_t* byte_strides, const int* box, bool fp32, bool swizzle128);
// 2-D map for epilogue stores: 32 x 32 boxes with 64-byte swizzle.
int make_tmap_2d_store(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                       int64_t ld);

}  // namespace cfb
