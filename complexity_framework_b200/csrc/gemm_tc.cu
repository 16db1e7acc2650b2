// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in tensor memory, operands staged by
// TMA into 128-byte-swizzled shared memory).
//
//   C[M,N] = epilogue( sum_k A(m,k) * B(n,k) )
//
// Operand storage (row-major, leading dimension in elements):
//   A K-major : A[M][lda]     (lda >= K)      A MN-major : A[K][lda] (lda >= M)
//   B K-major : B[N][ldb]     (ldb >= K)      B MN-major : B[K][ldb] (ldb >= N)
// so forward (X W^T), data-gradient (dY W) and weight-gradient (dY^T X) of a
// linear layer are all one kernel with different major flags, no transposes.
//
// CTA layout (256 threads, one CTA per SM, grid = #SMs, static tile striding):
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : TMEM allocator + MMA issuer (one elected lane)
//   warps 4..7  : epilogue warpgroup; warp w reads TMEM lanes 32*(w%4)..+31
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
//
// Epilogues fuse the elementwise work that follows each GEMM of the TR-Hash
// decoder layer: residual add (o_proj, MLP down), SwiGLU with the per-token
// routing weights of the deterministic experts (gate|up GEMM), the SwiGLU
// backward (data-gradient of the down projection), fp32 stores/accumulation
// for weight gradients, and per-tile softmax statistics for the fused LM-head
// cross-entropy.  Reference counterparts: the cuBLAS F.linear calls in
// complexity/core/attention/gqa.py:215-217,165 and
// complexity/tr_hash/engine.py:333-349, the Triton grouped GEMMs K4/K5/K7 of
// complexity_cuda/triton_token_routed.py:1031-1229,751-838 and the SwiGLU
// kernel K6 (:1232-1259).
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "gemm_tc.h"

namespace cfb {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;

// 32x32 bf16 staging boxes (2 KB) per epilogue warp: enough to keep each
// output of a column chunk in flight while the next chunk is converted.
__host__ __device__ constexpr int epi_slots(int epi) {
  return epi == EPI_SWIGLU_FWD ? 3
         : (epi == EPI_STORE || epi == EPI_RESID || epi == EPI_CE_STATS) ? 2 : 0;
}
// Epilogue operands read by TMA (32x32 bf16 boxes per column chunk): the
// residual for EPI_RESID, the saved gate and up pre-activations for
// EPI_SWIGLU_BWD.  Two chunks per warp are in flight (double buffer).
__host__ __device__ constexpr int epi_loads(int epi) {
  return epi == EPI_SWIGLU_BWD ? 2 : (epi == EPI_RESID ? 1 : 0);
}
// Column chunks of operand boxes in flight per warp.  EPI_SWIGLU_BWD stages
// its outputs in the consumed g/u boxes and stores them from there (no
// separate store slots), so the same shared memory holds three chunks.
__host__ __device__ constexpr int epi_depth(int epi) { return epi == EPI_SWIGLU_BWD ? 3 : 2; }
constexpr int kMaxLoadDepth = 4;
constexpr int kEpiWarps = 8;
constexpr int kBoxBytes = 32 * 32 * 2;
constexpr int kBarrierBytes = 512;

template <int BN, bool PAIR, int SLOTS, int LOADS = 0, int DEPTH = 2>
struct GemmCfg {
  // With PAIR, a 256-row tile is split over a CTA pair: each CTA holds its 128
  // A rows and half of the BN B rows; the even CTA issues M=256 MMAs.
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = B_ROWS * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int WARP_STAGING = (SLOTS + DEPTH * LOADS) * kBoxBytes;
  static constexpr int STAGING_BYTES = WARP_STAGING * kEpiWarps;
  static constexpr int STAGES = (227 * 1024 - 2048 - STAGING_BYTES) / STAGE_BYTES > 8
                                    ? 8
                                    : (227 * 1024 - 2048 - STAGING_BYTES) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int TILE_M = PAIR ? 2 * kBM : kBM;
  static constexpr int SMEM_BYTES =
      STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align*/ + kBarrierBytes;
};

// Lane `lane` writes row `lane` of a 32x32 bf16 box in the 64-byte-swizzled
// layout the store tensor map expects (16-byte unit q of row r sits at unit
// q ^ ((r >> 1) & 3)); eight consecutive lanes then hit distinct banks.
__device__ __forceinline__ void stage_row_bf16(uint8_t* box, int lane, const float* v,
                                               float alpha) {
  uint4* rowp = reinterpret_cast<uint4*>(box + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack_bf16x2(v[q * 8 + 0] * alpha, v[q * 8 + 1] * alpha);
    w.y = pack_bf16x2(v[q * 8 + 2] * alpha, v[q * 8 + 3] * alpha);
    w.z = pack_bf16x2(v[q * 8 + 4] * alpha, v[q * 8 + 5] * alpha);
    w.w = pack_bf16x2(v[q * 8 + 6] * alpha, v[q * 8 + 7] * alpha);
    rowp[q ^ sw] = w;
  }
}

// Per-warp ring of staging boxes written to global memory by TMA stores.
template <int SLOTS>
struct BoxRing {
  uint8_t* base;
  int slot;
  int lane;
  // stage one 32x32 box (this lane's row = v) and store it at (x, y)
  __device__ __forceinline__ void put(const CUtensorMap* map, const float* v, float alpha, int x,
                                      int y) {
    if (lane == 0) bulk_wait_group_read<SLOTS - 1>();  // the slot's previous store has read it
    __syncwarp();
    uint8_t* box = base + slot * kBoxBytes;
    stage_row_bf16(box, lane, v, alpha);
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, box, x, y);
      bulk_commit_group();
    }
    slot = slot + 1 == SLOTS ? 0 : slot + 1;
  }
  // two boxes staged together, one fence / sync / commit group (needs SLOTS >= 2)
  __device__ __forceinline__ void put2(const CUtensorMap* map, const float* v0, int x0,
                                       const float* v1, int x1, int y) {
    if (lane == 0) bulk_wait_group_read<SLOTS / 2 - 1>();  // previous pair has been read
    __syncwarp();
    uint8_t* b0 = base + slot * kBoxBytes;
    uint8_t* b1 = base + (slot + 1) * kBoxBytes;
    stage_row_bf16(b0, lane, v0, 1.0f);
    stage_row_bf16(b1, lane, v1, 1.0f);
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, b0, x0, y);
      tma_store_2d(map, b1, x1, y);
      bulk_commit_group();
    }
    slot = slot + 2 >= SLOTS ? 0 : slot + 2;
  }
};

// Row `lane` of a staged 32x32 bf16 box (64-byte swizzle, as written by TMA).
__device__ __forceinline__ void read_box_row(const uint8_t* box, int lane, float* v) {
  const uint4* rowp = reinterpret_cast<const uint4*>(box + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w = rowp[q ^ sw];
    const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z),
                 d = unpack_bf16x2(w.w);
    v[q * 8 + 0] = a.x; v[q * 8 + 1] = a.y; v[q * 8 + 2] = b.x; v[q * 8 + 3] = b.y;
    v[q * 8 + 4] = c.x; v[q * 8 + 5] = c.y; v[q * 8 + 6] = d.x; v[q * 8 + 7] = d.y;
  }
}

// Per-warp ring of TMA loads of epilogue operand boxes, DEPTH chunks deep.
// Tickets are issued and consumed in the same order; ticket k uses slot
// k % DEPTH and mbarrier phase (k / DEPTH) & 1.
template <int LOADS, int DEPTH = 2>
struct LoadRing {
  uint8_t* base;    // DEPTH slots x LOADS boxes
  uint64_t* bar;    // DEPTH mbarriers
  uint32_t issued;
  uint32_t consumed;
  int lane;
  __device__ __forceinline__ uint8_t* box(uint32_t ticket, int i) const {
    return base + ((ticket % DEPTH) * LOADS + i) * kBoxBytes;
  }
  // lane 0 issues the LOADS boxes at (xs[i], y)
  __device__ __forceinline__ void issue(const CUtensorMap* map, const int* xs, int y) {
    if (lane == 0) {
      uint64_t* b = &bar[issued % DEPTH];
      mbar_arrive_expect_tx(b, LOADS * kBoxBytes);
#pragma unroll
      for (int i = 0; i < LOADS; ++i) tma_load_2d(box(issued, i), map, b, xs[i], y);
    }
    ++issued;
  }
  __device__ __forceinline__ bool wait(volatile int* abort_flag, int* err) {
    const bool ok = mbar_wait(&bar[consumed % DEPTH], (consumed / DEPTH) & 1u, abort_flag, err,
                              kErrTimeoutFull, 14);
    return ok;
  }
  // every lane has read the consumed boxes; the slot may be refilled
  __device__ __forceinline__ void release() {
    __syncwarp();
    ++consumed;
  }
  // bounded wait for copies still in flight before the CTA exits
  __device__ __forceinline__ void drain(int* err) {
    while (consumed < issued) {
      mbar_wait(&bar[consumed % DEPTH], (consumed / DEPTH) & 1u, nullptr, err, kErrTimeoutFull,
                15);
      ++consumed;
    }
  }
};

// Scale that multiplies SwiGLU activation column `c` of row `row`.
__device__ __forceinline__ float swiglu_col_scale(const GemmEpi& ep, int row, int c) {
  if (c < ep.shared_width) return ep.shared_scale;
  int e = (c - ep.shared_width) / ep.expert_width;
  return ep.row_scale[static_cast<int64_t>(row) * ep.n_experts + e];
}

// Tensor maps of an operand: one map, or one per segment when the operand is
// the row-concatenation of per-rank shards (all-gather fused into the loads).
template <int NSEG>
struct SegMaps {
  CUtensorMap m[NSEG];
  int seg_rows;  // storage rows per segment (NSEG > 1)
  int nseg;
  // map holding storage row `row`, and the row inside that segment; rows past
  // the last segment stay out of range (TMA fills zeros)
  __device__ __forceinline__ const CUtensorMap* pick(int row, int* local) const {
    if constexpr (NSEG == 1) {
      *local = row;
      return &m[0];
    } else {
      int sidx = row / seg_rows;
      if (sidx >= nseg) sidx = nseg - 1;
      *local = row - sidx * seg_rows;
      return &m[sidx];
    }
  }
};

// One work unit of the persistent schedule: output tile t (row tile t / num_n),
// K blocks [kb0, kb1), group g.  Every role decodes the same units, so a unit
// without work is skipped by all of them (no loads, MMAs or epilogue hand-off).
struct Unit {
  int t, kb0, kb1, g;
  bool skip;
};

__device__ __forceinline__ Unit decode_unit(int u, int num_tiles, int num_n, int num_m,
                                            int m_shift, int ksplit, int nk, const GemmGroups& gr) {
  Unit r;
  if (gr.mode == 2) {
    const int per_group = num_tiles * ksplit;
    r.g = u / per_group;
    const int rem = u % per_group;
    r.t = rem / ksplit;
    const int s = rem % ksplit;
    const int g0 = __ldg(gr.k_start + r.g) / 64, g1 = __ldg(gr.k_start + r.g + 1) / 64;
    r.kb0 = g0 + s * (g1 - g0) / ksplit;
    r.kb1 = g0 + (s + 1) * (g1 - g0) / ksplit;
    r.skip = r.kb0 >= r.kb1;
    return r;
  }
  r.t = u / ksplit;
  r.kb0 = (u % ksplit) * nk / ksplit;
  r.kb1 = ((u % ksplit) + 1) * nk / ksplit;
  r.g = 0;
  r.skip = false;
  if (gr.mode == 1) {
    r.g = __ldg(gr.tile_group + (r.t / num_n + m_shift) % num_m);
    r.skip = r.g < 0;
  }
  return r;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool PAIR, int NA = 1, int NB = 1>
__global__ void __launch_bounds__(384, 1)
    gemm_tc_kernel(const __grid_constant__ SegMaps<NA> tmA,
                   const __grid_constant__ SegMaps<NB> tmB,
                   const __grid_constant__ CUtensorMap tmC0,
                   const __grid_constant__ CUtensorMap tmC1, int M, int N, int K, int ksplit,
                   GemmEpi ep, int* err) {
  constexpr int SLOTS = epi_slots(EPI);
  constexpr int LOADS = epi_loads(EPI);
  constexpr int DEPTH = epi_depth(EPI);
  using Cfg = GemmCfg<BN, PAIR, SLOTS, LOADS, DEPTH>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int B_ROWS = Cfg::B_ROWS;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint8_t* staging = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(staging + Cfg::STAGING_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* load_bar = tempty_bar + 2;  // kMaxLoadDepth per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(load_bar + kMaxLoadDepth * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;   // position inside the CTA pair
  const bool leader = rank == 0;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  const int num_m = (M + Cfg::TILE_M - 1) / Cfg::TILE_M;
  // with the fused all-gather, this rank's own row tiles come first
  const int m_shift = ep.ag.active ? (ep.sync.rank * ep.ag.rows) / Cfg::TILE_M : 0;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int nk = (K + kBK - 1) / kBK;
  // work unit u = (tile u / ksplit, K slice u % ksplit); ksplit > 1 only with the
  // fp32 atomic epilogue, which sums the partial products of the slices
  const int total = num_tiles * ksplit * (ep.grp.mode == 2 ? ep.grp.ngroups : 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      // one arrival per epilogue warp of every CTA in the MMA group
      mbar_init(&tempty_bar[a], PAIR ? 16 : 8);
    }
    for (int i = 0; i < kMaxLoadDepth * kEpiWarps; ++i) mbar_init(&load_bar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < (NA > 1 ? tmA.nseg : 1); ++i) tma_prefetch_desc(&tmA.m[i]);
    for (int i = 0; i < (NB > 1 ? tmB.nseg : 1); ++i) tma_prefetch_desc(&tmB.m[i]);
    // this rank's operand shard is complete (written by earlier kernels)
    if (ep.sync.world > 0 && ep.sync.signal && blockIdx.x == 0)
      sys_announce(ep.sync.pad, ep.sync.world, ep.sync.rank, ep.sync.round, ep.sync.epoch);
  }
  if (SLOTS > 0 && warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmC0);
    if (EPI == EPI_SWIGLU_FWD) tma_prefetch_desc(&tmC1);
  }
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    else
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync_all();  // peer barriers initialised before any remote arrive / TMA
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // operands in peer memory: every rank's shard must be written first
      if (ep.sync.world > 0 && ep.sync.role == 1)
        ok = sys_wait_all(ep.sync.pad, ep.sync.world, ep.sync.rank, ep.sync.round, ep.sync.epoch,
                          abort_flag, err, 16);
      for (int u = unit; u < total && ok; u += units) {
        const Unit un = decode_unit(u, num_tiles, num_n, num_m, m_shift, ksplit, nk, ep.grp);
        if (un.skip) continue;
        const int t = un.t, kb0 = un.kb0, kb1 = un.kb1;
        const int m0 = ((t / num_n + m_shift) % num_m) * Cfg::TILE_M + static_cast<int>(rank) * kBM;
        const int n0 = (t % num_n) * BN;
        // row-grouped: this group's B rows (K-major B) or K rows (MN-major B)
        const int b_off = ep.grp.mode == 1 ? static_cast<int>(un.g * ep.grp.b_stride) : 0;
        if (ep.ag.active) {
          // rows owned by a peer: wait until a copier warp has gathered them
          const int owner = m0 / ep.ag.rows;
          if (owner != ep.sync.rank && m0 < M) {
            const int* f = ep.ag.flags + m0 / kBM;
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_gpu(f) < ep.ag.epoch * (kBM / 16)) {
              if (*abort_flag || globaltimer_ns() - t0 > kWaitBoundNs) {
                if (!*abort_flag) report_error(err, kErrTimeoutFull, 19);
                *abort_flag = 1;
                ok = false;
                break;
              }
            }
            if (!ok) break;
            fence_proxy_async_all();  // gathered rows (generic stores) -> TMA reads
          }
        }
        // this CTA's B rows: half of the (possibly narrower) tail tile when paired
        const int n_rem = N - n0;
        const int n_this = n_rem < BN ? n_rem : BN;
        const int nb0 = (PAIR ? n0 + static_cast<int>(rank) * (n_this / 2) : n0) +
                        (B_MN ? 0 : b_off);
        const int kb_off = B_MN ? b_off : 0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, err, kErrTimeoutEmpty, 10)) {
            ok = false;
            break;
          }
          uint8_t* sA = tiles + stage * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          if constexpr (PAIR) {
            const uint32_t bar = mapa_shared(smem_u32(&full_bar[stage]), 0);
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
            int ra, rb;
            if constexpr (!A_MN) {
              const CUtensorMap* ma = tmA.pick(m0, &ra);
              tma_load_2d_pair(sA, ma, bar, kb * kBK, ra);
            } else {
              const CUtensorMap* ma = tmA.pick(kb * kBK, &ra);
#pragma unroll
              for (int i = 0; i < kBM / 64; ++i)
                tma_load_2d_pair(sA + i * 64 * kBK * 2, ma, bar, m0 + 64 * i, ra);
            }
            if constexpr (!B_MN) {
              const CUtensorMap* mb = tmB.pick(nb0, &rb);
              tma_load_2d_pair(sB, mb, bar, kb * kBK, rb);
            } else {
              const CUtensorMap* mb = tmB.pick(kb * kBK + kb_off, &rb);
#pragma unroll
              for (int i = 0; i < B_ROWS / 64; ++i)
                tma_load_2d_pair(sB + i * 64 * kBK * 2, mb, bar, nb0 + 64 * i, rb);
            }
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
            int ra, rb;
            if constexpr (!A_MN) {
              const CUtensorMap* ma = tmA.pick(m0, &ra);
              tma_load_2d(sA, ma, &full_bar[stage], kb * kBK, ra);
            } else {
              const CUtensorMap* ma = tmA.pick(kb * kBK, &ra);
#pragma unroll
              for (int i = 0; i < kBM / 64; ++i)
                tma_load_2d(sA + i * 64 * kBK * 2, ma, &full_bar[stage], m0 + 64 * i, ra);
            }
            if constexpr (!B_MN) {
              const CUtensorMap* mb = tmB.pick(nb0, &rb);
              tma_load_2d(sB, mb, &full_bar[stage], kb * kBK, rb);
            } else {
              const CUtensorMap* mb = tmB.pick(kb * kBK + kb_off, &rb);
#pragma unroll
              for (int i = 0; i < BN / 64; ++i)
                tma_load_2d(sB + i * 64 * kBK * 2, mb, &full_bar[stage], n0 + 64 * i, rb);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (leader && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = unit; u < total && ok; u += units) {
        const Unit un = decode_unit(u, num_tiles, num_n, num_m, m_shift, ksplit, nk, ep.grp);
        if (un.skip) continue;
        const int t = un.t, kb0 = un.kb0, kb1 = un.kb1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort_flag, err, kErrTimeoutTmem, 11)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        // the last column tile may be narrower than BN: issue a narrower MMA
        const int n_rem = N - (t % num_n) * BN;
        const uint32_t idesc = idesc_bf16(Cfg::TILE_M, n_rem < BN ? n_rem : BN, A_MN, B_MN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, err, kErrTimeoutFull, 12)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(tiles + stage * Cfg::STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = A_MN ? sw128_desc(a_base + k * 2048, 64 * kBK * 2, 1024)
                                        : sw128_desc(a_base + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? sw128_desc(b_base + k * 2048, 64 * kBK * 2, 1024)
                                        : sw128_desc(b_base + k * 32, 16, 1024);
            if constexpr (PAIR)
              umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
            else
              umma_bf16(d_tmem, adesc, bdesc, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          if constexpr (PAIR)
            umma_commit_pair(&empty_bar[stage], 0x3);
          else
            umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR)
          umma_commit_pair(&tfull_bar[acc], 0x3);
        else
          umma_commit(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ all-gather copiers
    // two warps per CTA pull 128-row chunks of the peers' shards over NVLink
    // (8 x 16-byte loads in flight per lane) into this rank's gathered buffer
    if (ep.ag.active) {
      bool ok = true;
      if (ep.sync.world > 0 && lane == 0)
        ok = sys_wait_all(ep.sync.pad, ep.sync.world, ep.sync.rank, ep.sync.round,
                          ep.sync.epoch, abort_flag, err, 20);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      // work unit = 16-row piece of a 128-row chunk; a chunk is complete when
      // its counter has grown by kPieces in this epoch
      constexpr int kPieceRows = 16, kPieces = kBM / kPieceRows;
      const int chunks_per_rank = ep.ag.rows / kBM;
      const int world = ep.sync.world;
      const int remote = (world - 1) * chunks_per_rank * kPieces;
      const int64_t piece_elems = static_cast<int64_t>(kPieceRows) * ep.ag.cols;
      const int64_t n16 = piece_elems / 8;
      const int copier = 2 * static_cast<int>(blockIdx.x) + (warp - 2);
      const int copiers = 2 * static_cast<int>(gridDim.x);
      for (int j = copier; ok && j < remote; j += copiers) {
        // pieces in the order the producers consume chunks: peers' rows after own
        const int jc = j / kPieces, jp = j % kPieces;
        const int q = (ep.sync.rank + 1 + jc / chunks_per_rank) % world;
        const int chunk = q * chunks_per_rank + jc % chunks_per_rank;
        const int64_t off = (static_cast<int64_t>(chunk) * kPieces + jp) * piece_elems;
        const uint4* src = reinterpret_cast<const uint4*>(ep.ag.src[q] + off);
        uint4* dst = reinterpret_cast<uint4*>(ep.ag.dst + off);
        int64_t i = lane;
        for (; i + 15 * 32 < n16; i += 16 * 32) {
          uint4 r[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) r[k] = src[i + k * 32];
#pragma unroll
          for (int k = 0; k < 16; ++k) dst[i + k * 32] = r[k];
        }
        for (; i < n16; i += 32) dst[i] = src[i];
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          fence_proxy_async_all();
          atomicAdd(ep.ag.flags + chunk, 1);  // release: fenced above
        }
        if (*abort_flag) break;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // two epilogue warpgroups (warps 4-7 and 8-11) split the tile's columns;
    // warp w reads TMEM lanes 32*(w%4)..+31, i.e. rows of the tile
    const int wq = warp & 3;
    const int wg = (warp - 4) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t tempty_peer0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
    const uint32_t tempty_peer1 = mapa_shared(smem_u32(&tempty_bar[1]), 0);
    uint8_t* wstage = staging + (warp - 4) * Cfg::WARP_STAGING;
    BoxRing<SLOTS ? SLOTS : 1> ring{wstage, 0, lane};
    LoadRing<LOADS ? LOADS : 1, DEPTH> lring{wstage + SLOTS * kBoxBytes,
                                              load_bar + kMaxLoadDepth * (warp - 4), 0u,
                                      0u, lane};
    bool ep_ok = true;
    for (int u = unit; u < total; u += units) {
      const Unit un = decode_unit(u, num_tiles, num_n, num_m, m_shift, ksplit, nk, ep.grp);
      if (un.skip) continue;
      const int t = un.t;
      // K-grouped weight gradients: this group's output rows
      const int64_t c_row0 = ep.grp.mode == 2 ? un.g * ep.grp.c_stride : 0;
      const int m_blk = (t / num_n + m_shift) % num_m;
      const int n_blk = t % num_n;
      const int m0 = m_blk * Cfg::TILE_M + static_cast<int>(rank) * kBM;
      const int n0 = n_blk * BN;
      // operand boxes of the warp's first column chunk load while the MMA runs
      const int cbeg = wg * (BN / 2);
      if constexpr (EPI == EPI_SWIGLU_BWD) {
        if (n0 + cbeg < N) {
          const int ac = n0 + cbeg;
          const int xs[2] = {(ac / kSwigluBlock) * 2 * kSwigluBlock + ac % kSwigluBlock,
                             (ac / kSwigluBlock) * 2 * kSwigluBlock + ac % kSwigluBlock +
                                 kSwigluBlock};
          if (lane == 0) bulk_wait_group_read<0>();  // see the chunk loop
          __syncwarp();
          lring.issue(&tmC1, xs, m0 + wq * 32);
          if (n0 + cbeg + 32 < N) {  // and the second chunk: loads run two chunks ahead
            const int ac2 = ac + 32;
            const int xs2[2] = {(ac2 / kSwigluBlock) * 2 * kSwigluBlock + ac2 % kSwigluBlock,
                                (ac2 / kSwigluBlock) * 2 * kSwigluBlock + ac2 % kSwigluBlock +
                                    kSwigluBlock};
            lring.issue(&tmC1, xs2, m0 + wq * 32);
          }
        }
      } else if constexpr (EPI == EPI_RESID) {
        if (n0 + cbeg < N) {
          const int xs[1] = {n0 + cbeg};
          lring.issue(&tmC1, xs, m0 + wq * 32);
        }
      }
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, err, kErrTimeoutTmem, 13)) break;
      tc_fence_after();
      const int row = m0 + wq * 32 + lane;
      const bool row_ok = row < M;
      const uint32_t tbase = tmem_base + acc * BN + (static_cast<uint32_t>(wq * 32) << 16);

      if constexpr (EPI == EPI_SWIGLU_FWD) {
        // Tile columns [0, BN/2) are gate, [BN/2, BN) are the matching up columns.
        constexpr int HALF = BN / 2;
#pragma unroll 1
        for (int c = wg * HALF / 2; c < (wg + 1) * HALF / 2; c += 32) {
          float g[32], u[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + HALF + c, u);
          tmem_wait_ld();
          const int act_col = n_blk * HALF + c;
          if (n0 + c < N) {  // warp-uniform; rows >= M are clipped by the stores
            const int y = m0 + wq * 32;
            ring.put(&tmC0, g, 1.0f, n0 + c, y);
            ring.put(&tmC0, u, 1.0f, n0 + HALF + c, y);
            const float s = row_ok ? swiglu_col_scale(ep, row, act_col) : 0.0f;
            float a[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              // Round the pre-activations to bf16 first so that forward and the
              // recomputation in backward see identical inputs.
              const float gb = __bfloat162float(__float2bfloat16(g[i]));
              const float ub = __bfloat162float(__float2bfloat16(u[i]));
              a[i] = silu_f(gb) * ub * s;
            }
            ring.put(&tmC1, a, 1.0f, act_col, y);
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU_BWD) {
        // Accumulator = d(act) for activation columns [n0, n0+BN); the saved
        // pre-activations g, u arrive in shared memory by TMA (prefetched).
#pragma unroll 1
        for (int c = cbeg; c < cbeg + BN / 2; c += 32) {
          const int act_col = n0 + c;
          if (act_col >= N) break;  // warp-uniform; later chunks are out of range too
          if (c + 64 < cbeg + BN / 2 && act_col + 64 < N) {
            const int ac = act_col + 64;
            const int xs[2] = {(ac / kSwigluBlock) * 2 * kSwigluBlock + ac % kSwigluBlock,
                               (ac / kSwigluBlock) * 2 * kSwigluBlock + ac % kSwigluBlock +
                                   kSwigluBlock};
            // loads run two chunks ahead: the slot refilled for chunk c+2 last
            // held chunk c-1's outputs, whose store must have read it
            if (lane == 0) bulk_wait_group_read<0>();
            __syncwarp();
            lring.issue(&tmC1, xs, m0 + wq * 32);
          }
          float da[32];
          tmem_ld32(tbase + c, da);
          tmem_wait_ld();
          if (!lring.wait(abort_flag, err)) {
            ep_ok = false;
            break;
          }
          uint8_t* gbox = lring.box(lring.consumed, 0);
          uint8_t* ubox = lring.box(lring.consumed, 1);
          float g[32], u[32];
          read_box_row(gbox, lane, g);
          read_box_row(ubox, lane, u);
          const int blk = act_col / kSwigluBlock;
          const int w = act_col % kSwigluBlock;
          const float s = row_ok ? swiglu_col_scale(ep, row, act_col) : 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float sg = sigmoid_f(g[i]);
            const float d = da[i] * s;
            const float du = d * g[i] * sg;
            g[i] = d * u[i] * sg * (1.0f + g[i] * (1.0f - sg));  // d(gate)
            u[i] = du;                                          // d(up)
          }
          // outputs go out from the boxes the inputs came in (each lane
          // rewrites only the row it read)
          stage_row_bf16(gbox, lane, g, 1.0f);
          stage_row_bf16(ubox, lane, u, 1.0f);
          fence_proxy_async_shared();
          __syncwarp();
          const int x = blk * 2 * kSwigluBlock + w;
          if (lane == 0) {
            tma_store_2d(&tmC0, gbox, x, m0 + wq * 32);
            tma_store_2d(&tmC0, ubox, x + kSwigluBlock, m0 + wq * 32);
            bulk_commit_group();
          }
          ++lring.consumed;
        }
        if (!ep_ok) break;
      } else if constexpr (EPI == EPI_CE_STATS) {
        // Store bf16 logits and, per (row, n-tile), the max and sum(exp(x-max)).
        float mx = -INFINITY, se = 0.0f;
#pragma unroll 1
        for (int c = wg * BN / 2; c < (wg + 1) * BN / 2; c += 32) {
          float v[32];
          tmem_ld32(tbase + c, v);
          tmem_wait_ld();
          if (n0 + c < N) {  // warp-uniform
            float lm = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v[i] = __bfloat162float(__float2bfloat16(v[i] * ep.alpha));
              if (n0 + c + i < N) lm = fmaxf(lm, v[i]);
            }
            const float nm = fmaxf(mx, lm);
            float acc_e = se * __expf(mx - nm);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (n0 + c + i < N) acc_e += __expf(v[i] - nm);
            mx = nm;
            se = acc_e;
            ring.put(&tmC0, v, 1.0f, n0 + c, m0 + wq * 32);
          }
        }
        if (row_ok) {
          float2* st = reinterpret_cast<float2*>(ep.stats);
          // one (max, sumexp) pair per half tile (BN/2 columns)
          st[static_cast<int64_t>(row) * num_n * 2 + n_blk * 2 + wg] = make_float2(mx, se);
        }
      } else {
#pragma unroll 1
        for (int c = wg * BN / 2; c < (wg + 1) * BN / 2; c += 32) {
          float r[32];
          if constexpr (EPI == EPI_RESID) {
            if (n0 + c >= N) break;  // warp-uniform
            if (c + 32 < (wg + 1) * BN / 2 && n0 + c + 32 < N) {
              const int xs[1] = {n0 + c + 32};
              lring.issue(&tmC1, xs, m0 + wq * 32);
            }
          }
          float v[32];
          tmem_ld32(tbase + c, v);
          tmem_wait_ld();
          if constexpr (EPI == EPI_STORE) {
            if (n0 + c < N) ring.put(&tmC0, v, ep.alpha, n0 + c, m0 + wq * 32);
          } else if constexpr (EPI == EPI_RESID) {
            if (!lring.wait(abort_flag, err)) {
              ep_ok = false;
              break;
            }
            read_box_row(lring.box(lring.consumed, 0), lane, r);
            lring.release();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = v[i] * ep.alpha + r[i];
            ring.put(&tmC0, v, 1.0f, n0 + c, m0 + wq * 32);
          } else if (row_ok && n0 + c < N) {
            if constexpr (EPI == EPI_PEER_STORE) {
              // this rank's partial rows go to the owner's slot for this rank
              const int owner = static_cast<int>(row / ep.peer_rows);
              const int64_t lrow = row - static_cast<int64_t>(owner) * ep.peer_rows;
              float4* out = reinterpret_cast<float4*>(
                  ep.peer_c[owner] +
                  (static_cast<int64_t>(ep.sync.rank) * ep.peer_rows + lrow) * ep.ldc + n0 + c);
#pragma unroll
              for (int q = 0; q < 8; ++q)
                out[q] = make_float4(v[4 * q] * ep.alpha, v[4 * q + 1] * ep.alpha,
                                     v[4 * q + 2] * ep.alpha, v[4 * q + 3] * ep.alpha);
            } else if constexpr (EPI == EPI_F32_ATOMIC) {
              float* out = reinterpret_cast<float*>(ep.c) + (c_row0 + row) * ep.ldc + n0 + c;
#pragma unroll
              for (int q = 0; q < 8; ++q)
                red_add_v4(out + 4 * q, v[4 * q] * ep.alpha, v[4 * q + 1] * ep.alpha,
                           v[4 * q + 2] * ep.alpha, v[4 * q + 3] * ep.alpha);
            } else if constexpr (EPI == EPI_F32 || EPI == EPI_F32_ACC) {
              float4* out = reinterpret_cast<float4*>(reinterpret_cast<float*>(ep.c) +
                                                      static_cast<int64_t>(row) * ep.ldc + n0 + c);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 w = make_float4(v[4 * q] * ep.alpha, v[4 * q + 1] * ep.alpha,
                                       v[4 * q + 2] * ep.alpha, v[4 * q + 3] * ep.alpha);
                if constexpr (EPI == EPI_F32_ACC) {
                  float4 o = out[q];
                  w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
                }
                out[q] = w;
              }
            }
          }
        }
        if (!ep_ok) break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(acc ? tempty_peer1 : tempty_peer0);
        else
          mbar_arrive(&tempty_bar[acc]);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (LOADS > 0) lring.drain(err);
    if ((SLOTS > 0 || EPI == EPI_SWIGLU_BWD) && lane == 0) bulk_wait_group_all();
    if constexpr (EPI == EPI_PEER_STORE) __threadfence_system();  // peer stores before exit
  }

  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync_all();  // both CTAs' epilogues are done before the pair frees TMEM
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
// cuTensorMapEncodeTiled is a driver call: it fails with CUDA_ERROR_INVALID_CONTEXT
// on a host thread that has no current context yet (a fresh thread whose only
// CUDA work so far was served from PyTorch's caching allocator, e.g. the
// autograd engine's worker thread).  Make the current device's primary context
// current on such threads first.
// Driver entry points are looked up through the runtime, so the extension has
// no link-time dependency on libcuda (it imports on machines without a driver).
void ensure_current_context() {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  static GetCurrentFn get_current = nullptr;
  if (get_current == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q);
    get_current = reinterpret_cast<GetCurrentFn>(p);
  }
  CUcontext ctx = nullptr;
  if (get_current != nullptr && get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr) return;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  ensure_current_context();
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

// Map a row-major bf16 matrix [rows][ld] (inner extent `cols`) as 2-D tiles of
// box_inner x box_outer with 128-byte swizzle.
int make_tmap_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                 int box_inner, int box_outer) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r) + 1000;
}

// Generic tiled map: `rank` dims (innermost first), byte strides of dims 1..rank-1,
// element type bf16 (fp32 = false) or fp32, 128-byte swizzle or none.  Rows
// outside the tensor read as zero.
int make_tmap_nd(CUtensorMap* map, const void* base, int rank, const int64_t* dims,
                 const int64_t* byte_strides, const int* box, bool fp32, bool swizzle128) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return -1;
  if (rank < 1 || rank > 5) return -2;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = static_cast<cuuint64_t>(dims[i]);
    bx[i] = static_cast<cuuint32_t>(box[i]);
    es[i] = 1;
    if (i > 0) st[i - 1] = static_cast<cuuint64_t>(byte_strides[i - 1]);
  }
  CUresult r = fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                  static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r) + 1000;
}

int make_tmap_2d_store(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                       int64_t ld) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r) + 1000;
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool PAIR, int NA = 1, int NB = 1>
static int launch_impl(const SegMaps<NA>& ta, const SegMaps<NB>& tb, const CUtensorMap* tc,
                       int M, int N, int K, const GemmEpi& ep, int num_sms, cudaStream_t stream,
                       int* err, int ksplit = 1) {
  using Cfg = GemmCfg<BN, PAIR, epi_slots(EPI), epi_loads(EPI), epi_depth(EPI)>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, EPI, PAIR, NA, NB>;
  static int max_units = -1;  // resident CTAs (or CTA pairs), one query per instantiation
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(384, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_units < 0) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (PAIR) {
      cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0)
        clusters = num_sms / 2;
      max_units = clusters;
    } else {
      max_units = num_sms;
    }
  }
  // K-grouped weight gradients: every group contributes its own tiles; its K
  // range is about K / groups on average
  const int groups = ep.grp.mode == 2 ? ep.grp.ngroups : 1;
  const int tiles = ((M + Cfg::TILE_M - 1) / Cfg::TILE_M) * ((N + BN - 1) / BN) * groups;
  if (EPI == EPI_F32_ATOMIC && ksplit == 0) {
    // pick the K split that fills the machine best (>= 8 K blocks per slice)
    const int nk = (K / groups + kBK - 1) / kBK;
    int best = 1;
    double best_eff = 0.0;
    for (int ks = 1; ks <= 16 && nk / ks >= 8; ++ks) {
      const int work = tiles * ks;
      const int waves = (work + max_units - 1) / max_units;
      const double eff = static_cast<double>(work) / (static_cast<double>(waves) * max_units);
      if (eff > best_eff + 0.02) {
        best_eff = eff;
        best = ks;
      }
    }
    ksplit = best;
  }
  if (ksplit < 1) ksplit = 1;
  const int work = tiles * ksplit;
  const int units = work < max_units ? work : max_units;
  cfg.gridDim = dim3(PAIR ? 2 * units : units, 1, 1);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc[0], tc[1], M, N, K, ksplit, ep, err);
  return static_cast<int>(e);
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static int launch_pair_or_single(const SegMaps<1>& ta, const SegMaps<1>& tb, const CUtensorMap* tc,
                                 int M, int N, int K, const GemmEpi& ep, int sms, cudaStream_t s,
                                 int* err) {
  const int ks = EPI == EPI_F32_ATOMIC ? 0 : 1;  // 0 = choose
  // 256-row tiles over an SM pair halve each SM's operand traffic per FLOP;
  // a single 128-row tile is used only when M itself fits in one.
  // (keep in sync with the B tensor-map box chosen in gemm_tc_launch)
  if (M > kBM) return launch_impl<BN, A_MN, B_MN, EPI, true>(ta, tb, tc, M, N, K, ep, sms, s, err, ks);
  return launch_impl<BN, A_MN, B_MN, EPI, false>(ta, tb, tc, M, N, K, ep, sms, s, err, ks);
}

template <int BN, int EPI>
static int dispatch_major(bool a_mn, bool b_mn, const SegMaps<1>& ta, const SegMaps<1>& tb,
                          const CUtensorMap* tc, int M, int N, int K, const GemmEpi& ep, int sms,
                          cudaStream_t s, int* err) {
  if (!a_mn && !b_mn)
    return launch_pair_or_single<BN, false, false, EPI>(ta, tb, tc, M, N, K, ep, sms, s, err);
  if (!a_mn && b_mn)
    return launch_pair_or_single<BN, false, true, EPI>(ta, tb, tc, M, N, K, ep, sms, s, err);
  if (a_mn && !b_mn)
    return launch_pair_or_single<BN, true, false, EPI>(ta, tb, tc, M, N, K, ep, sms, s, err);
  return launch_pair_or_single<BN, true, true, EPI>(ta, tb, tc, M, N, K, ep, sms, s, err);
}

int choose_bn(int M, int N, int num_sms) {
  (void)M;
  (void)num_sms;
  return N <= 128 ? 128 : 256;
}

// Operand tensor maps.  `rows` x `cols` is the storage shape of one map.
static int make_operand_map(CUtensorMap* map, const void* base, bool mn, int64_t rows, int64_t cols,
                            int64_t ld, int box_rows_kmajor) {
  return mn ? make_tmap_2d(map, base, rows, cols, ld, 64, kBK)
            : make_tmap_2d(map, base, rows, cols, ld, kBK, box_rows_kmajor);
}

static int epilogue_maps(const GemmArgs& g, const GemmEpi& ep, CUtensorMap* tc) {
  // epilogue store maps (bf16 outputs written by TMA from staging boxes)
  memset(tc, 0, 2 * sizeof(CUtensorMap));
  int rc = 0;
  switch (g.epi) {
    case EPI_STORE:
    case EPI_CE_STATS:
      rc = make_tmap_2d_store(&tc[0], ep.c, g.M, g.N, ep.ldc);
      break;
    case EPI_RESID:
      rc = make_tmap_2d_store(&tc[0], ep.c, g.M, g.N, ep.ldc);
      if (!rc) rc = make_tmap_2d_store(&tc[1], ep.r, g.M, g.N, ep.ldr);  // residual loads
      break;
    case EPI_SWIGLU_FWD:
      rc = make_tmap_2d_store(&tc[0], ep.gu, g.M, g.N, ep.ldgu);
      if (!rc) rc = make_tmap_2d_store(&tc[1], ep.act, g.M, g.N / 2, ep.ldact);
      break;
    case EPI_SWIGLU_BWD: {
      int64_t cols = 2 * static_cast<int64_t>((g.N + kSwigluBlock - 1) / kSwigluBlock) * kSwigluBlock;
      if (cols > ep.ldc) cols = ep.ldc;
      rc = make_tmap_2d_store(&tc[0], ep.c, g.M, cols, ep.ldc);
      int64_t gcols = 2 * static_cast<int64_t>((g.N + kSwigluBlock - 1) / kSwigluBlock) *
                      kSwigluBlock;
      if (gcols > ep.ldgu) gcols = ep.ldgu;
      if (!rc) rc = make_tmap_2d_store(&tc[1], ep.gu, g.M, gcols, ep.ldgu);  // g/u loads
      break;
    }
    default:
      break;
  }
  return rc;
}

// Distributed variants (tensor parallel): all-gather fused into the operand
// loads (segmented A or B) and reduce-scatter by peer stores.  256-row CTA
// pairs, BN = 256.
static int gemm_tc_launch_dist(const GemmArgs& g, const GemmEpi& ep, cudaStream_t stream,
                               int* err) {
  if (g.M <= kBM) return -6;
  const int box_b = 256 / 2;
  CUtensorMap tc[2];
  int rc = epilogue_maps(g, ep, tc);
  if (rc) return rc;
  const int ks = g.epi == EPI_F32_ATOMIC ? 0 : 1;
  if (g.a_nseg > 0) {
    if (g.a_nseg > kMaxSeg || g.a_seg_rows % (g.a_mn ? kBK : kBM) != 0) return -7;
    SegMaps<kMaxSeg> sa;
    memset(&sa, 0, sizeof(sa));
    sa.seg_rows = static_cast<int>(g.a_seg_rows);
    sa.nseg = g.a_nseg;
    for (int i = 0; i < g.a_nseg; ++i) {
      rc = make_operand_map(&sa.m[i], g.A_seg[i], g.a_mn, g.a_seg_rows, g.a_mn ? g.M : g.K, g.lda,
                            kBM);
      if (rc) return rc;
    }
    SegMaps<1> sb;
    rc = g.b_mn ? make_operand_map(&sb.m[0], g.B, true, g.K, g.N, g.ldb, box_b)
                : make_operand_map(&sb.m[0], g.B, false, g.N, g.K, g.ldb, box_b);
    if (rc) return rc;
    sb.seg_rows = 0;
    sb.nseg = 1;
#define CFB_DIST_A(AM, BM, E)                                                                   \
  if (g.a_mn == AM && g.b_mn == BM && g.epi == E)                                               \
    return launch_impl<256, AM, BM, E, true, kMaxSeg, 1>(sa, sb, tc, g.M, g.N, g.K, ep,        \
                                                          g.num_sms, stream, err, ks);
    CFB_DIST_A(false, false, EPI_STORE)
    CFB_DIST_A(false, false, EPI_SWIGLU_FWD)
    CFB_DIST_A(false, true, EPI_STORE)
    CFB_DIST_A(false, true, EPI_SWIGLU_BWD)
    CFB_DIST_A(true, true, EPI_F32_ATOMIC)
#undef CFB_DIST_A
    return -8;
  }
  if (g.b_nseg > 0) {
    if (g.b_nseg > kMaxSeg || !g.b_mn || g.b_seg_rows % kBK != 0) return -7;
    SegMaps<1> sa;
    rc = g.a_mn ? make_operand_map(&sa.m[0], g.A, true, g.K, g.M, g.lda, kBM)
                : make_operand_map(&sa.m[0], g.A, false, g.M, g.K, g.lda, kBM);
    if (rc) return rc;
    sa.seg_rows = 0;
    sa.nseg = 1;
    SegMaps<kMaxSeg> sb;
    memset(&sb, 0, sizeof(sb));
    sb.seg_rows = static_cast<int>(g.b_seg_rows);
    sb.nseg = g.b_nseg;
    for (int i = 0; i < g.b_nseg; ++i) {
      rc = make_operand_map(&sb.m[i], g.B_seg[i], true, g.b_seg_rows, g.N, g.ldb, box_b);
      if (rc) return rc;
    }
    if (g.a_mn && g.epi == EPI_F32_ATOMIC)
      return launch_impl<256, true, true, EPI_F32_ATOMIC, true, 1, kMaxSeg>(
          sa, sb, tc, g.M, g.N, g.K, ep, g.num_sms, stream, err, ks);
    return -8;
  }
  // reduce-scatter: plain operands, peer-store epilogue
  if (g.epi != EPI_PEER_STORE || ep.peer_rows <= 0) return -8;
  SegMaps<1> sa, sb;
  rc = g.a_mn ? make_operand_map(&sa.m[0], g.A, true, g.K, g.M, g.lda, kBM)
              : make_operand_map(&sa.m[0], g.A, false, g.M, g.K, g.lda, kBM);
  if (rc) return rc;
  rc = g.b_mn ? make_operand_map(&sb.m[0], g.B, true, g.K, g.N, g.ldb, box_b)
              : make_operand_map(&sb.m[0], g.B, false, g.N, g.K, g.ldb, box_b);
  if (rc) return rc;
  sa.seg_rows = sb.seg_rows = 0;
  sa.nseg = sb.nseg = 1;
  if (g.a_mn) return -8;
  if (g.b_mn)
    return launch_impl<256, false, true, EPI_PEER_STORE, true>(sa, sb, tc, g.M, g.N, g.K, ep,
                                                                 g.num_sms, stream, err, 1);
  return launch_impl<256, false, false, EPI_PEER_STORE, true>(sa, sb, tc, g.M, g.N, g.K, ep,
                                                                g.num_sms, stream, err, 1);
}

int gemm_tc_launch(const GemmArgs& g, const GemmEpi& ep, cudaStream_t stream, int* err) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return -2;
  if (g.a_nseg > 0 || g.b_nseg > 0 || g.epi == EPI_PEER_STORE)
    return gemm_tc_launch_dist(g, ep, stream, err);
  int bn = g.bn;
  if (g.epi == EPI_SWIGLU_FWD) bn = 2 * kSwigluBlock;
  if (bn == 0) {
    bn = choose_bn(g.M, g.N, g.num_sms);
    // split-K weight gradients with N an odd multiple of 128 (896, 1152 here):
    // 128-column tiles leave no half-empty tile and measured 6-17% faster
    if (g.epi == EPI_F32_ATOMIC && g.N % 256 != 0 && g.N % 128 == 0) bn = 128;
  }
  if (bn != 128 && bn != 256) return -3;
  SegMaps<1> ta, tb;
  ta.seg_rows = tb.seg_rows = 0;
  ta.nseg = tb.nseg = 1;
  if (ep.grp.mode == 1 && (ep.grp.tile_group == nullptr || ep.grp.ngroups <= 0 ||
                           ep.grp.b_stride <= 0 || g.M % 256 != 0))
    return -9;
  if (ep.grp.mode == 2 && (ep.grp.k_start == nullptr || ep.grp.ngroups <= 0 || !g.a_mn ||
                           !g.b_mn || g.epi != EPI_F32_ATOMIC))
    return -9;
  int rc = g.a_mn ? make_operand_map(&ta.m[0], g.A, true, g.K, g.M, g.lda, kBM)
                  : make_operand_map(&ta.m[0], g.A, false, g.M, g.K, g.lda, kBM);
  if (rc) return rc;
  // row-grouped: B holds every group's rows
  const int64_t b_rows = ep.grp.mode == 1 ? ep.grp.ngroups * ep.grp.b_stride : -1;
  // pair mode: each CTA loads half of a K-major B tile
  rc = g.b_mn ? make_operand_map(&tb.m[0], g.B, true, b_rows > 0 ? b_rows : g.K, g.N, g.ldb, bn)
              : make_operand_map(&tb.m[0], g.B, false, b_rows > 0 ? b_rows : g.N, g.K, g.ldb,
                                 g.M > kBM ? bn / 2 : bn);
  if (rc) return rc;
  CUtensorMap tc[2];
  rc = epilogue_maps(g, ep, tc);
  if (rc) return rc;

#define CFB_EPI_CASE(E)                                                                          \
  case E:                                                                                        \
    return bn == 256 ? dispatch_major<256, E>(g.a_mn, g.b_mn, ta, tb, tc, g.M, g.N, g.K, ep,      \
                                              g.num_sms, stream, err)                            \
                     : dispatch_major<128, E>(g.a_mn, g.b_mn, ta, tb, tc, g.M, g.N, g.K, ep,      \
                                              g.num_sms, stream, err);
  switch (g.epi) {
    CFB_EPI_CASE(EPI_STORE)
    CFB_EPI_CASE(EPI_RESID)
    CFB_EPI_CASE(EPI_F32)
    CFB_EPI_CASE(EPI_F32_ACC)
    CFB_EPI_CASE(EPI_F32_ATOMIC)
    CFB_EPI_CASE(EPI_CE_STATS)
    case EPI_SWIGLU_FWD:
      if (g.a_mn || g.b_mn) return -4;
      return launch_pair_or_single<256, false, false, EPI_SWIGLU_FWD>(ta, tb, tc, g.M, g.N, g.K, ep,
                                                                      g.num_sms, stream, err);
    case EPI_SWIGLU_BWD:
      if (g.a_mn || !g.b_mn) return -4;
      return bn == 256 ? launch_pair_or_single<256, false, true, EPI_SWIGLU_BWD>(
                             ta, tb, tc, g.M, g.N, g.K, ep, g.num_sms, stream, err)
                       : launch_pair_or_single<128, false, true, EPI_SWIGLU_BWD>(
                             ta, tb, tc, g.M, g.N, g.K, ep, g.num_sms, stream, err);
    default:
      return -5;
  }
#undef CFB_EPI_CASE
}

}  // namespace cfb
