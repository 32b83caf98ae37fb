// NVFP4 block-scaled GEMM and dual GEMM (fused SiLU gate) for sm_100a.
//
//   GEMM:  C[m,n,l] = fp16( sum_k (A sfA)[m,k,l] (B sfB)[n,k,l] )
//          ref_kernel of problems/nvidia/nvfp4_gemm/reference.py:27-53
//   Dual:  C[m,n,l] = fp16( silu(A.B1^T) * (A.B2^T) ), both products in fp32
//          ref_kernel of problems/nvidia/nvfp4_dual_gemm/reference.py:27-77
//
// Structure (one CTA per SM, persistent, 10 warps):
//   warp 0      TMA producer: A/B tiles with 128-byte swizzle through
//               cp.async.bulk.tensor, the 128x4-blocked scale factors through
//               plain cp.async.bulk (each 128-row block of scales for a
//               256-wide K tile is one contiguous 2 KB run), into a ring of
//               kStages shared-memory stages guarded by full/empty mbarriers.
//   warps 6..9  scale copiers, one per TMEM lane quarter: per K tile each
//               reads the stage's scale blocks from shared memory and writes
//               them into its 32 TMEM lanes with tcgen05.st (the blocks
//               replicated to the four lane quarters, the layout the MMA
//               reads), then arrives on full[stage].  tcgen05.cp of the
//               same blocks costs ~45 tensor-pipe cycles each and competes
//               with the MMAs for the pipe (measured); the stores do not.
//   warp 1      TMEM owner and MMA issuer: per K tile, four tcgen05.mma
//               kind::mxf4nvf4 (M=128, N=BN, K=64 each; for the dual GEMM
//               N=256 over the adjacent B1 and B2 tiles, so A is read once
//               for both products) accumulate in fp32 in TMEM;
//               tcgen05.commit releases the stage and, after the last K tile,
//               hands the accumulator to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld rows of the accumulator(s), optional
//               silu(x)*y in fp32, fp16 conversion, 16-byte global stores.
// With BN=128 the GEMM double-buffers its accumulator in TMEM so the epilogue
// of tile i overlaps the main loop of tile i+1; BN=256 and the dual GEMM need
// all accumulator columns for one tile.  No load uses cluster multicast.
#include "common.cuh"
#include "kernels.h"

#include <cmath>
#include <cstdlib>
#include <mutex>

namespace nvfp4 {

// Optional per-CTA timing of the pipeline waits (build with -DNVFP4_TRACE;
// read with nvfp4_dbg_gemm_trace).  Slots per CTA: 0 MMA waiting for a stage,
// 1 MMA waiting for its scales, 2 MMA role total, 3 producer waiting for a
// free stage, 4 scale writer waiting for a stage, 5 scale writer total,
// 6 epilogue waiting for an accumulator, 7 epilogue total (SM cycles).
#ifdef NVFP4_TRACE
__device__ unsigned long long g_gemm_trace[1024 * 32];
// Slots 8.. hold %globaltimer stamps: 8 kernel entry, 9 after setup and the
// PDL wait, 10 last accumulator handed to the epilogue, 11 epilogue done,
// 12 kernel exit.
#define TRACE_STAMP(slot) g_gemm_trace[blockIdx.x * 32 + (slot)] = global_timer_ns()
// Slot 13: SM cycles the MMA thread spends issuing (MMAs + commit, after its waits).
// Slots 14, 15: clock64 of thread 0 at the stamps of slots 9 and 12 (SM MHz).
#define TRACE_CLOCK(slot) \
  if (threadIdx.x == 0) g_gemm_trace[blockIdx.x * 32 + (slot)] = clock64()
#define TRACE_ISSUE_BEGIN const long long _ti0 = clock64()
#define TRACE_ISSUE_END trace[13] += clock64() - _ti0
#define TRW(slot, expr)                      \
  ({                                         \
    const long long _t0 = clock64();         \
    const bool _r = (expr);                  \
    trace[slot] += clock64() - _t0;          \
    _r;                                      \
  })
#define TRACE_DECL unsigned long long trace[20] = {}; const long long trace_t0 = clock64()
#define TRACE_TOTAL(slot) trace[slot] = clock64() - trace_t0
#define TRACE_FLUSH()                                                             \
  do {                                                                            \
    if (lane == 0)                                                                \
      for (int _i = 0; _i < 20; ++_i)                                             \
        if (trace[_i]) g_gemm_trace[blockIdx.x * 32 + _i] = trace[_i];             \
  } while (0)
#else
#define TRW(slot, expr) (expr)
#define TRACE_DECL
#define TRACE_TOTAL(slot)
#define TRACE_FLUSH()
#define TRACE_STAMP(slot)
#define TRACE_ISSUE_BEGIN
#define TRACE_ISSUE_END
#define TRACE_CLOCK(slot)
#endif

constexpr int kBM = 128;
constexpr int kBK = 256;          // K elements per stage (128 bytes per row)
constexpr int kBKBytes = kBK / 2;
constexpr int kMmaK = 64;         // K per tcgen05.mma for kind::mxf4nvf4
constexpr int kStreamKFlagBytes = 4096;  // stream-K flags at the workspace start (<= 1024 CTAs)
constexpr int kSfBlockBytes = 512;  // one 128-row x 4-scale block
constexpr int kSfStageBytes = kSfBlockBytes * (kBK / kMmaK);  // 2 KB per operand per stage
// Scale copiers of the 1-CTA kernel: four warps (6..9), one per TMEM lane
// quarter, write the scales with tcgen05.st.
constexpr int kCopiers = 4;
// TMA producers: warp 0 and warps 10.. .  A thread that waits on an mbarrier
// between its bulk copies keeps only about one copy in flight (measured: one
// producer thread streams ~60 GB/s into an SM whatever the ring depth, four
// reach ~130 GB/s per SM with every SM loading), so the K tiles are dealt
// round-robin to kProducers warps, each waiting only for its own stages.
#ifndef NVFP4_PRODUCERS
#define NVFP4_PRODUCERS 4
#endif
constexpr int kProducers = NVFP4_PRODUCERS;
constexpr int kThreads = 192 + 32 * kCopiers + 32 * (kProducers - 1);
// The 2-CTA kernel: four scale-writer warps per CTA as well.
constexpr int kPairCopiers = 4;
constexpr int kPairThreads = 192 + 32 * kPairCopiers + 32 * (kProducers - 1);

// Producer index of a warp (0 .. kProducers-1), or -1.
__device__ __forceinline__ int producer_index(int warp) {
  return warp == 0 ? 0 : (warp >= 10 && warp < 9 + kProducers) ? warp - 9 : -1;
}

template <int BN, bool kDual>
struct GemmConfig {
  static constexpr int kNB = kDual ? 2 : 1;  // number of B operands
  static constexpr int kABytes = kBM * kBKBytes;
  static constexpr int kBBytes = BN * kBKBytes;
  static constexpr int kStageBytes = kABytes + kNB * kBBytes;
  static constexpr int kSfOps = 1 + kNB * (BN / 128);                // 2 KB scale runs per stage
  static constexpr int kStages = (kDual || BN == 256) ? 4 : 5;
  static constexpr int kAccBufs = (kDual || BN == 256) ? 1 : 2;
  static constexpr int kAccCols = kNB * BN;                           // fp32 columns per accumulator buffer
  static constexpr int kSfCols = 16 * kSfOps;                         // TMEM columns of scales per stage
  static constexpr int kTmemCols = 512;
  static_assert(kAccBufs * kAccCols + kStages * kSfCols <= kTmemCols, "TMEM budget");
  // A producer waits on empty[stage] by phase parity, which is only exact
  // while no stage can be two laps ahead of the MMA; a producer's previous
  // wait (K tile g - kProducers) covers K tile g - kProducers - kStages, so
  // that holds only when kProducers <= kStages.
  static_assert(kProducers <= kStages, "more producer warps than stages breaks the parity waits");
  static constexpr int kTxBytes = kStageBytes;                 // full[]: A and B tiles
  static constexpr int kSmemBytes =
      1024 /*align slack*/ + kStages * (kStageBytes + kSfOps * kSfStageBytes) + 256 /*barriers*/;
};

struct GemmParams {
  const uint8_t* sfa;   // blocked scales of A, batch l at sfa + l * sfa_lstride
  const uint8_t* sfb;   // blocked scales of B (B1 for the dual GEMM)
  const uint8_t* sfb2;  // blocked scales of B2 (dual GEMM only)
  __half* c;
  int M, N, K, L;
  int64_t sfa_lstride, sfb_lstride, sfb2_lstride;  // bytes
  int64_t ldc, c_lstride;                          // elements
  int tiles_m, tiles_n, num_tiles;
  int group_m;  // raster: groups of group_m M-blocks sweep all N-blocks
  int inject;   // test hook: 1 = CTA 0 withholds its first A load (its pipeline waits then run out)
  int splits;   // K splits per tile (1 = none); work item = tile * splits + split.
                // With splits > 1 the kernel is launched with clusters of
                // `splits` CTAs, one item per CTA, cluster = tile.
  int num_items;
  int prefetch;  // K tiles ahead to prefetch B into L2 (0 = off)
  int b_evict;   // L2 policy of B loads: 0 evict_first, 1 evict_normal, 2 evict_last
  // Stream-K (splits == 1 only): the tiles x K-tiles "units", in tile-major
  // order, are cut into gridDim.x equal contiguous ranges, one per CTA.  A CTA
  // whose range starts inside a tile (its first segment) writes that partial
  // tile, fp32, to slot blockIdx.x of sk_partial and raises sk_flag[blockIdx.x];
  // the CTA holding the tile's first K tiles (its last segment) adds the
  // partials of the following CTAs, in CTA order, and writes C.
  // Hybrid form: tiles [0, dp_tiles) are whole work items dealt round-robin
  // (dp_tiles a multiple of the worker count, the full waves), and only the
  // remaining tiles' units are cut into the equal ranges, so the full waves
  // keep the classic lockstep order over K (the tiles sharing an A or B slice
  // read it at about the same time, from L2).
  int streamk;
  int dp_tiles;
  int64_t units;  // units of the split tiles [dp_tiles, num_tiles)
  float* sk_partial;  // gridDim.x slots of kBM x BN floats
  int* sk_flag;       // gridDim.x flags, 0 between launches
  int* status;
};

// MMA K steps (of 64) in K tile kt: 4, or fewer in a partial last tile.
__device__ __forceinline__ int ksteps(int K, int kt) {
  const int r = (K - kt * 256) / 64;
  return r < 4 ? r : 4;
}

// Bytes of one 128-row block's scale run in K tile kt (2 KB, less in a partial tile).
__device__ __forceinline__ uint32_t sf_run_bytes(int K, int kt) { return static_cast<uint32_t>(ksteps(K, kt)) * 512u; }

// K-tile range [k0, k1) of split s.
__device__ __forceinline__ void split_range(int KT, int splits, int s, int& k0, int& k1) {
  k0 = (s * KT) / splits;
  k1 = ((s + 1) * KT) / splits;
}

// First unit of worker b's stream-K range (nw workers: CTAs, or CTA pairs).
__device__ __forceinline__ int64_t sk_begin(const GemmParams& p, int b, int nw) {
  return (static_cast<int64_t>(b) * p.units) / nw;
}

// The work items of worker w of nw (a CTA, or a CTA pair), in order: (tile,
// K-tile range).  Every warp role walks the same sequence.
struct WorkIter {
  int64_t u, u_end;
  int it, nw, dp_t;
  __device__ __forceinline__ WorkIter(const GemmParams& p, int w, int nw_) {
    it = w;
    nw = nw_;
    u = p.streamk ? sk_begin(p, w, nw) : 0;
    u_end = p.streamk ? sk_begin(p, w + 1, nw) : 0;
    dp_t = (p.streamk && w < p.dp_tiles) ? w : -1;  // whole tiles first
  }
  __device__ __forceinline__ bool next(const GemmParams& p, int KT, int& t, int& k0, int& k1) {
    if (p.streamk) {
      if (dp_t >= 0) {
        t = dp_t;
        k0 = 0;
        k1 = KT;
        dp_t = (dp_t + nw < p.dp_tiles) ? dp_t + nw : -1;
        return true;
      }
      if (u >= u_end) return false;
      const int ts = static_cast<int>(u / KT);
      t = p.dp_tiles + ts;
      k0 = static_cast<int>(u - static_cast<int64_t>(ts) * KT);
      const int64_t rem = u_end - u;
      k1 = (KT - k0 > rem) ? k0 + static_cast<int>(rem) : KT;
      u += k1 - k0;
      return true;
    }
    if (it >= p.num_items) return false;
    t = it / p.splits;
    split_range(KT, p.splits, it - t * p.splits, k0, k1);
    it += nw;
    return true;
  }
};

// Whether worker c has a non-empty stream-K range (ranges are empty when the
// split tiles have fewer units than there are workers).
__device__ __forceinline__ bool sk_has_range(const GemmParams& p, int c, int nw) {
  return sk_begin(p, c, nw) < sk_begin(p, c + 1, nw);
}

// End (exclusive, in stream-K units) of split tile t.
__device__ __forceinline__ int64_t sk_tile_end(const GemmParams& p, int t, int KT) {
  return static_cast<int64_t>(t - p.dp_tiles + 1) * KT;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// AND of `pred` over the 128 epilogue threads (named barrier 1).
__device__ __forceinline__ bool epi_all(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return out != 0;
}

__device__ __forceinline__ void set_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& mb, int& nb, int& l) {
  const int per_l = p.tiles_m * p.tiles_n;
  l = t / per_l;
  int r = t - l * per_l;
  const int group_size = p.group_m * p.tiles_n;
  const int g = r / group_size;
  const int first_m = g * p.group_m;
  const int gm = min(p.tiles_m - first_m, p.group_m);
  r -= g * group_size;
  mb = first_m + r % gm;
  nb = r / gm;
}

__device__ __forceinline__ float silu_mul(float x, float y) {
  return __fdividef(x, 1.0f + __expf(-x)) * y;
}

// 32 fp32 values -> fp16, four 16-byte stores.
__device__ __forceinline__ void store_half_row32(__half* dst_row, const uint32_t (&r)[32]) {
  uint4 out[4];
  uint32_t* o = reinterpret_cast<uint32_t*>(out);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    __half2 h = __floats2half2_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    o[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  uint4* dst = reinterpret_cast<uint4*>(dst_row);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = out[i];
}

// For the four epilogue warps, the AND of `flag` over them (named barrier 1);
// other warps get true without touching the barrier.
__device__ __forceinline__ bool epi_all_maybe(bool is_epi, bool flag) {
  return is_epi ? epi_all(flag) : true;
}

// Cluster-wide barrier (every thread of every CTA in the cluster), with
// release/acquire ordering of shared::cluster accesses.
__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_peer(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Column groups (32 output columns each) [g0, g1) owned by split rank s of S.
__device__ __forceinline__ void share_groups(int ngroups, int S, int s, int& g0, int& g1) {
  g0 = (s * ngroups) / S;
  g1 = ((s + 1) * ngroups) / S;
}

template <int BN, bool kDual>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_b2, const __grid_constant__ CUtensorMap tm_c,
                const GemmParams p) {
  if (threadIdx.x == 0) TRACE_STAMP(8);
  using Cfg = GemmConfig<BN, kDual>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;                                   // S x kStageBytes (1024-aligned each)
  uint8_t* sfbuf = smem + S * Cfg::kStageBytes;            // S x kSfOps x 2 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sfbuf + S * Cfg::kSfOps * kSfStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* sf_full = bars + 3 * S;  // the stage's scale runs landed (before its A/B tiles, usually)
  uint64_t* acc_full = bars + 4 * S;
  uint64_t* acc_empty = acc_full + Cfg::kAccBufs;
  uint64_t* drain = acc_empty + Cfg::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = (p.K + kBK - 1) / kBK;  // the last K tile may be partial (K % 64 == 0)

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      // full: the producer's expect-tx arrival, the A/B bytes, and one
      // arrival per scale writer warp once the stage's scales are in TMEM
      // (the MMA thread waits on this one barrier per K tile).
      mbar_init(&full[s], 1 + kCopiers);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_full[s], 1);
    }
    for (int b = 0; b < Cfg::kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
    if (kDual) prefetch_tensormap(&tm_b2);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t sf_col0 = Cfg::kAccBufs * Cfg::kAccCols;
  if (threadIdx.x == 0) pdl_allow_dependents();
  pdl_wait();
  TRACE_DECL;
  if (threadIdx.x == 0) TRACE_STAMP(9);
  TRACE_CLOCK(14);
  bool split_ready = false;  // epilogue threads: this CTA's split partial is in TMEM

  if (producer_index(warp) >= 0) {
    // ------------------------------------------------------------ producers
    // K tile g of this CTA's sequence (over all its work items) goes to
    // producer g % kProducers, in stage g % S.
    const int pidx = producer_index(warp);
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_of(p.b_evict);
      int g = 0;
      WorkIter wi(p, blockIdx.x, gridDim.x);
      int t, k0, k1, item = 0;
      for (; !abort_flag && wi.next(p, KT, t, k0, k1); ++item) {
        int mb, nb, l;
        tile_coords(p, t, mb, nb, l);
        const uint8_t* sfa_src = p.sfa + l * p.sfa_lstride + static_cast<int64_t>(mb) * p.K * 8;
        const uint8_t* sfb_src = p.sfb + l * p.sfb_lstride + static_cast<int64_t>(nb) * (BN / 128) * p.K * 8;
        const uint8_t* sfb2_src =
            kDual ? p.sfb2 + l * p.sfb2_lstride + static_cast<int64_t>(nb) * (BN / 128) * p.K * 8 : nullptr;
        for (int kt = k0; kt < k1; ++kt, ++g) {
          if (g % kProducers != pidx) continue;
          const int stage = g % S;
          const uint32_t phase = (g / S) & 1;
          if (!TRW(3, mbar_wait(&empty[stage], phase ^ 1))) {
            set_status(p.status, kStatusTimeoutEmpty);
            abort_flag = 1;
            break;
          }
          uint8_t* st = tiles + stage * Cfg::kStageBytes;
          uint8_t* sf = sfbuf + stage * Cfg::kSfOps * kSfStageBytes;
          // Scales first, on their own barrier: the writers can put them in
          // TMEM while the larger A/B tiles are still arriving.
          const uint32_t sfb_bytes = sf_run_bytes(p.K, kt);
          mbar_arrive_expect_tx(&sf_full[stage], Cfg::kSfOps * sfb_bytes);
          bulk_load(sf, sfa_src + kt * kSfStageBytes, sfb_bytes, &sf_full[stage], pol_a);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            bulk_load(sf + (1 + j) * kSfStageBytes, sfb_src + static_cast<int64_t>(j) * p.K * 8 + kt * kSfStageBytes,
                      sfb_bytes, &sf_full[stage], pol_b);
          if (kDual) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              bulk_load(sf + (1 + BN / 128 + j) * kSfStageBytes,
                        sfb2_src + static_cast<int64_t>(j) * p.K * 8 + kt * kSfStageBytes, sfb_bytes,
                        &sf_full[stage], pol_b);
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kTxBytes);
          if (!(p.inject && blockIdx.x == 0 && item == 0 && kt == k0))
            tma_load_3d(st, &tm_a, &full[stage], kt * kBKBytes, mb * kBM, l, pol_a);
          tma_load_3d(st + Cfg::kABytes, &tm_b, &full[stage], kt * kBKBytes, nb * BN, l, pol_b);
          if (kDual) tma_load_3d(st + Cfg::kABytes + Cfg::kBBytes, &tm_b2, &full[stage], kt * kBKBytes, nb * BN, l, pol_b);
          // L2 prefetch of the B tiles p.prefetch K tiles ahead (beyond the
          // shared-memory ring): more DRAM requests in flight for shapes that
          // stream B from DRAM.
          if (p.prefetch && kt + p.prefetch < k1) {
            tma_prefetch_3d(&tm_b, (kt + p.prefetch) * kBKBytes, nb * BN, l);
            if (kDual) tma_prefetch_3d(&tm_b2, (kt + p.prefetch) * kBKBytes, nb * BN, l);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kBM, BN);
      constexpr uint32_t idesc_dual = idesc_nvf4(kBM, 2 * BN);
      static_assert(!kDual || BN == 128, "dual GEMM: B1|B2 form one N=256 operand");
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      WorkIter wi(p, blockIdx.x, gridDim.x);
      int t, k0, k1;
      while (!abort_flag && wi.next(p, KT, t, k0, k1)) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) {
          set_status(p.status, kStatusTimeoutAccEmpty);
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * Cfg::kAccCols;
        bool ok = true;
        for (int kt = k0; kt < k1; ++kt) {
          if (!TRW(0, mbar_wait(&full[stage], phase))) {
            set_status(p.status, kStatusTimeoutFull);
            abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          TRACE_ISSUE_BEGIN;
          const uint32_t st = smem_u32(tiles + stage * Cfg::kStageBytes);
          const uint32_t sfc = tmem_base + sf_col0 + stage * Cfg::kSfCols;
          const int nkk = ksteps(p.K, kt);
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk) {
            if (kk >= nkk) break;
            const uint64_t adesc = desc_kmajor_sw128(st + kk * (kMmaK / 2));
            const uint64_t bdesc = desc_kmajor_sw128(st + Cfg::kABytes + kk * (kMmaK / 2));
            const uint32_t accum = (kt != k0 || kk != 0) ? 1u : 0u;
            if (kDual) {
              // The B1 and B2 tiles sit back to back in shared memory: one
              // N=2*BN MMA (B2 as rows BN.. of B) reads A once for both
              // products; accumulator columns [0,BN) = A.B1, [BN,2BN) = A.B2.
              mma_nvf4(d0, adesc, bdesc, idesc_dual, sfc + 4 * kk, sfc + 16 + 8 * kk, accum);
            } else {
              mma_nvf4(d0, adesc, bdesc, idesc, sfc + 4 * kk, sfc + 16 + 4 * kk * (BN / 128), accum);
            }
          }
          tc_commit(&empty[stage]);
          TRACE_ISSUE_END;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
        TRACE_STAMP(10);
        if (++acc == Cfg::kAccBufs) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Make sure every issued tcgen05 op has retired before TMEM is freed.
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp >= 6 && warp <= 9) {
    // ------------------------------------------------------------ scale copiers
    // Warps 6..9, one per TMEM lane quarter (warp % 4).  Per stage every
    // warp reads the stage's 512-byte scale blocks from shared memory (lane
    // i takes the 16 bytes of rows i, i+32, i+64, i+96) and writes them with
    // tcgen05.st to its 32 lanes, four columns per block: together the four
    // warps leave TMEM exactly as tcgen05.cp.32x128b.warpx4 would (the
    // block replicated to all four lane quarters).  Layout per stage: SFA
    // at columns [0,16) (MMA step kk at 4*kk), then the B scales: 128-row
    // block j of step kk at 16 + 4*(kk*NB + j), NB = 128-row blocks per MMA
    // (BN/128, or 2 for the dual GEMM's B1|B2), the order an N=128*NB MMA
    // reads them in.
    // tcgen05.st does not enter the tensor pipe, so unlike tcgen05.cp
    // (~45 pipe cycles per block) it does not take issue slots from the MMAs.
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    int total = 0;
    {
      WorkIter wi(p, blockIdx.x, gridDim.x);
      int t, k0, k1;
      while (wi.next(p, KT, t, k0, k1)) total += k1 - k0;
    }
    for (int i = 0; i < total; ++i) {
      const bool got = TRW(4, mbar_wait(&sf_full[stage], phase));
      if (!__all_sync(0xffffffffu, got && !abort_flag)) {
        if (lane == 0 && !got) set_status(p.status, kStatusTimeoutFull);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint8_t* sf = sfbuf + stage * Cfg::kSfOps * kSfStageBytes + lane * 16;
      const uint32_t sfc = tmem_base + lane_base + sf_col0 + stage * Cfg::kSfCols;
#pragma unroll
      for (int r = 0; r < Cfg::kSfOps; ++r)
#pragma unroll
        for (int kk = 0; kk < kBK / kMmaK; ++kk) {
          const uint4 v = *reinterpret_cast<const uint4*>(sf + r * kSfStageBytes + kk * kSfBlockBytes);
          // Dual: B1 and B2 are the two 128-row blocks of one N=256 operand.
          const int col = r == 0  ? 4 * kk
                          : kDual ? 16 + 4 * (2 * kk + (r - 1))
                                  : 16 + 4 * (kk * (BN / 128) + (r - 1) % (BN / 128));
          tmem_st_32x32b_x4(sfc + col, v);
        }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[stage]);
      if (++stage == S) {
        stage = 0;
        phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool split = p.splits > 1;
    WorkIter wi(p, blockIdx.x, gridDim.x);
    int t, k0, k1;
    while (wi.next(p, KT, t, k0, k1)) {
      int mb, nb, l;
      tile_coords(p, t, mb, nb, l);
      // All lanes (and, with split K, all four epilogue warps, which meet at
      // named barriers below) must agree before the collective tcgen05.ld.
      const bool got = TRW(6, mbar_wait(&acc_full[acc], acc_phase));
      if (split ? !epi_all(got) : !__all_sync(0xffffffffu, got)) {
        if (lane == 0) set_status(p.status, kStatusTimeoutAccFull);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int rloc = q * 32 + lane;
      const int row = mb * kBM + rloc;
      __half* crow = p.c + l * p.c_lstride + static_cast<int64_t>(row) * p.ldc + static_cast<int64_t>(nb) * BN;
      const uint32_t tacc = tmem_base + acc * Cfg::kAccCols + (static_cast<uint32_t>(q * 32) << 16);
      if (!kDual && !split && p.streamk && k0 > 0) {
        // Stream-K contributor: this CTA holds K tiles [k0, k1) of tile t
        // (the first segment of its range).  Partial sums go to its slot as
        // [column group][float4 index][row][4], one coalesced 512-byte row
        // of float4 per warp instruction; then the flag is raised.
        float4* dst = reinterpret_cast<float4*>(p.sk_partial) + static_cast<int64_t>(blockIdx.x) * (kBM * BN / 4) + rloc;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tacc + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[((c0 / 32) * 8 + i) * kBM] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                                         __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        epi_bar();
        if (threadIdx.x == 64) {
          __threadfence();
          st_release_gpu(p.sk_flag + blockIdx.x, 1);
        }
      } else if (!split) {
        // Stream-K finaliser (K tiles [0, k1) with k1 < KT, the last segment
        // of this CTA's range): the rest of the tile was computed by the
        // following CTAs [blockIdx.x + 1, c_end) as their first segments.
        int c_end = blockIdx.x + 1;
        if (p.streamk && k1 < KT) {
          const int64_t tile_end = sk_tile_end(p, t, KT);
          while (c_end < static_cast<int>(gridDim.x) && sk_begin(p, c_end, gridDim.x) < tile_end) ++c_end;
          bool ok = true;
          if (threadIdx.x == 64) {
            for (int c = blockIdx.x + 1; c < c_end && ok; ++c)
              if (sk_has_range(p, c, gridDim.x)) ok = flag_wait(p.sk_flag + c);
            if (ok)
              for (int c = blockIdx.x + 1; c < c_end; ++c) p.sk_flag[c] = 0;  // ready for the next launch
            else
              set_status(p.status, kStatusTimeoutPeer);
          }
          if (!epi_all(ok)) {
            abort_flag = 1;
            break;
          }
        }
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tacc + c0, r);
          if (kDual) {
            uint32_t r2[32];
            tmem_ld_32x32b_x32(tacc + BN + c0, r2);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              r[i] = __float_as_uint(silu_mul(__uint_as_float(r[i]), __uint_as_float(r2[i])));
          } else {
            tmem_wait_ld();
            // Own partial first, then the contributors' in CTA order: the
            // same order on every call with the same grid.
            for (int c = blockIdx.x + 1; c < c_end; ++c) {
              if (!sk_has_range(p, c, gridDim.x)) continue;
              const float4* src = reinterpret_cast<const float4*>(p.sk_partial) +
                                  static_cast<int64_t>(c) * (kBM * BN / 4) + (c0 / 32) * 8 * kBM + rloc;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 v = __ldcg(src + i * kBM);
                r[4 * i] = __float_as_uint(__uint_as_float(r[4 * i]) + v.x);
                r[4 * i + 1] = __float_as_uint(__uint_as_float(r[4 * i + 1]) + v.y);
                r[4 * i + 2] = __float_as_uint(__uint_as_float(r[4 * i + 2]) + v.z);
                r[4 * i + 3] = __float_as_uint(__uint_as_float(r[4 * i + 3]) + v.w);
              }
            }
          }
          store_half_row32(crow + c0, r);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
      } else {
        // Split K: one item per CTA; the accumulator stays in TMEM for the
        // cluster exchange below.
        split_ready = true;
      }
      if (++acc == Cfg::kAccBufs) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  if (p.splits > 1) {
    // ---------------------------------------------------------- split-K reduction
    // The CTAs of a cluster hold the partial sums of one tile for different K
    // ranges.  Columns are cut into S shares (groups of 32 output columns, with
    // both accumulators of a group for the dual GEMM); rank r writes its
    // partials of every other rank's share straight into that rank's shared
    // memory (st.shared::cluster), then each rank adds the partials of its own
    // share in rank order (identical on every call) and writes C.  The
    // pipeline shared memory is reused as the receive buffer, so the first
    // cluster barrier waits until every rank's main loop is done with it.
    constexpr int NG = BN / 32;
    constexpr int GF = 32 * Cfg::kNB;  // floats per row per group
    const int S = p.splits;
    const int rank = static_cast<int>(cluster_ctarank());
    const int t = blockIdx.x / S;
    const int max_share = (NG + S - 1) / S;
    const bool epi = warp >= 2 && warp <= 5;
    const bool ok = epi_all_maybe(epi, split_ready);
    tc_fence_after();
    cluster_sync_all();  // every rank: main loop finished, smem free
    const int q = warp & 3;
    const int rloc = q * 32 + lane;
    const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    // recv[slot][group][f4][row][4 floats], slot = sender rank minus one if above us
    auto recv_off = [&](int slot, int gi, int f4) -> uint32_t {
      return static_cast<uint32_t>((((slot * max_share + gi) * (GF / 4) + f4) * kBM + rloc) * 16);
    };
    if (epi && ok) {
      const uint32_t base = smem_u32(tiles);
      for (int peer = 0; peer < S; ++peer) {
        if (peer == rank) continue;
        const uint32_t pbase = map_peer(base, static_cast<uint32_t>(peer));
        const int slot = rank < peer ? rank : rank - 1;
        int g0, g1;
        share_groups(NG, S, peer, g0, g1);
        for (int g = g0; g < g1; ++g) {
#pragma unroll
          for (int b = 0; b < Cfg::kNB; ++b) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tacc + b * BN + g * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i)
              st_cluster_v4(pbase + recv_off(slot, g - g0, b * 8 + i), __uint_as_float(r[4 * i]),
                            __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                            __uint_as_float(r[4 * i + 3]));
          }
        }
      }
    }
    cluster_sync_all();  // all partials delivered
    if (epi && ok) {
      int mb, nb, l;
      tile_coords(p, t, mb, nb, l);
      // This rank's share of C, 32-column groups of 128 rows x 64 bytes,
      // staged after the receive slots and written by TMA stores (one box
      // per group; measured the same speed as 64-byte row pieces stored by
      // every thread, and the stores leave the SM as a few bulk requests).
      const uint32_t recv_bytes = static_cast<uint32_t>((S - 1) * max_share * (GF / 4) * kBM * 16);
      uint8_t* out_stage = tiles + ((recv_bytes + 1023u) & ~1023u);
      int g0, g1;
      share_groups(NG, S, rank, g0, g1);
      const float4* recv = reinterpret_cast<const float4*>(tiles);
      for (int g = g0; g < g1; ++g) {
        // Own partial first, then the received ones in slot (rank) order:
        // the same rank owns the same columns on every call, so the order of
        // the additions, and the result, is the same on every call.
        float acc[Cfg::kNB][32];
#pragma unroll
        for (int b = 0; b < Cfg::kNB; ++b) {
          uint32_t own[32];
          tmem_ld_32x32b_x32(tacc + b * BN + g * 32, own);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc[b][i] = __uint_as_float(own[i]);
        }
        const float4* src = recv + ((g - g0) * (GF / 4)) * kBM + rloc;
        for (int slot = 0; slot < S - 1; ++slot, src += max_share * (GF / 4) * kBM) {
#pragma unroll
          for (int b = 0; b < Cfg::kNB; ++b) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 v = src[(b * 8 + i) * kBM];
              acc[b][4 * i] += v.x;
              acc[b][4 * i + 1] += v.y;
              acc[b][4 * i + 2] += v.z;
              acc[b][4 * i + 3] += v.w;
            }
          }
        }
        uint32_t res[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          res[i] = __float_as_uint(kDual ? silu_mul(acc[0][i], acc[Cfg::kNB - 1][i]) : acc[0][i]);
        uint4* dst = reinterpret_cast<uint4*>(out_stage + (g - g0) * (kBM * 64) + rloc * 64);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __half2 h0 = __floats2half2_rn(__uint_as_float(res[8 * j + 0]), __uint_as_float(res[8 * j + 1]));
          __half2 h1 = __floats2half2_rn(__uint_as_float(res[8 * j + 2]), __uint_as_float(res[8 * j + 3]));
          __half2 h2 = __floats2half2_rn(__uint_as_float(res[8 * j + 4]), __uint_as_float(res[8 * j + 5]));
          __half2 h3 = __floats2half2_rn(__uint_as_float(res[8 * j + 6]), __uint_as_float(res[8 * j + 7]));
          dst[j] = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                              *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
        }
      }
      fence_proxy_async_smem();
      epi_bar();
      if (threadIdx.x == 64) {
        for (int g = g0; g < g1; ++g)
          tma_store_3d(&tm_c, out_stage + (g - g0) * (kBM * 64), (nb * BN + g * 32) * 2, mb * kBM, l);
        bulk_commit_group();
        bulk_wait_group0();  // complete before the CTA exits
      }
    }
  }

#ifdef NVFP4_TRACE
  if (threadIdx.x == 64) TRACE_STAMP(11);
  if (warp == 1) TRACE_TOTAL(2);
  if (warp == 6) TRACE_TOTAL(5);
  if (warp == 2) TRACE_TOTAL(7);
  if (warp <= 2 || warp == 6) TRACE_FLUSH();
#endif
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0) TRACE_STAMP(12);
  TRACE_CLOCK(15);
}

// ------------------------------------------------------------------ 2-CTA GEMM
// Pairs of CTAs (a cluster of 2) compute 256x256 tiles with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=64): each CTA loads its own 128
// rows of A and its own 128 rows of B (half of the tile's N), so per output
// element each SM streams half the B bytes of the single-CTA 128x256 tile and
// its shared memory sees 32 KB of TMA writes and 32 KB of MMA reads per K tile
// instead of 48 + 48 KB.  Scale factors: each CTA holds SFA for its 128 rows
// and SFB for all 256 columns in its own TMEM, written by its own four
// writer warps (tcgen05.st) from its own shared memory.  A and B loads signal
// the leader's full barrier (.cta_group::2 TMA); the writers of both CTAs
// arrive on the leader's full barrier; MMA completion is multicast to
// both CTAs' empty / accumulator barriers.  No load uses cluster multicast.
namespace pair {
constexpr int kStages = 4;
constexpr int kA = kBM * kBKBytes;       // 16 KB: this CTA's 128 rows of A
constexpr int kB = 128 * kBKBytes;       // 16 KB: this CTA's 128 rows of B
constexpr int kSfa = kSfStageBytes;      // 2 KB
constexpr int kSfb = 2 * kSfStageBytes;  // 4 KB: both 128-row blocks of the tile's N
constexpr int kStage = kA + kB + kSfa + kSfb;
constexpr int kTx = 2 * (kA + kB);  // the leader's full barrier counts both CTAs' A and B bytes
constexpr int kAccCols = 256;
constexpr int kSfCols = 48;
constexpr int kTmemCols = 512;
static_assert(kAccCols + kStages * kSfCols <= kTmemCols, "TMEM budget");
static_assert(kProducers <= kStages, "more producer warps than stages breaks the parity waits");
static_assert(kStage % 1024 == 0, "stage alignment");
constexpr int kFixBufs = 8;          // stream-K finaliser ring: 8 x 16 KB in the stage area
constexpr int kFixChunk = 16 * 1024;  // one (contributor, 32-column group) of a partial slot
constexpr int kMaxContrib = 16;       // contributors per finalised tile
static_assert(kFixBufs * kFixChunk <= kStages * kStage, "fix-up ring fits in the stage area");
// Epilogue staging for whole tiles: this CTA's 128 x 256 fp16 outputs as four
// 64-column boxes of 128 rows x 128 bytes (128-byte swizzle), written from
// TMEM by the epilogue warps and stored to C by TMA while the next tile's
// MMAs run (the accumulator is released as soon as TMEM has been read).
constexpr int kOutBox = 128 * 128;
constexpr int kOut = 4 * kOutBox;
constexpr int kSmem = 1024 + kStages * kStage + kOut + 256;
static_assert(kSmem <= 227 * 1024, "shared memory budget");
}  // namespace pair

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t mbar_cluster, int x,
                                                 int y, int z, uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(mbar_cluster), "l"(hint)
      : "memory");
}

__device__ __forceinline__ void mma_nvf4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Arrive on the barrier at this offset in the CTAs of `mask` when this
// thread's prior cta_group::2 tcgen05 operations complete.
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// kDual: the dual GEMM on 256 x (128 B1 + 128 B2) tiles: CTA 0 loads the B1
// tile and CTA 1 the B2 tile, which together form the N=256 operand, so the
// accumulator row of either CTA holds A.B1 in columns [0,128) and A.B2 in
// [128,256) and the SiLU gate is applied per CTA.
template <bool kDual>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_b2, const __grid_constant__ CUtensorMap tm_c,
                     const GemmParams p) {
  if (threadIdx.x == 0) TRACE_STAMP(8);
  using namespace pair;
  constexpr int S = kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* outbuf = smem + S * kStage;  // epilogue staging (kOut bytes, 1024-aligned)
  uint64_t* bars = reinterpret_cast<uint64_t*>(outbuf + kOut);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* sf_full = bars + 3 * S;
  uint64_t* acc_full = bars + 4 * S;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;  // MMA thread
  uint64_t* fix_full = drain + 1;   // stream-K finaliser: kFixBufs partial-chunk buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fix_full + kFixBufs);
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = (p.K + kBK - 1) / kBK;  // the last K tile may be partial (K % 64 == 0)
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      // The leader's full: its producer's expect-tx arrival, both CTAs' A/B
      // bytes, and the scale writer warps of both CTAs (one wait per K tile
      // for the MMA thread).
      mbar_init(&full[s], 1 + 2 * kPairCopiers);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_full[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * 128);
    mbar_init(drain, 1);
    for (int i = 0; i < kFixBufs; ++i) mbar_init(&fix_full[i], 1);
    fence_barrier_init();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(kDual && rank ? &tm_b2 : &tm_b);
    prefetch_tensormap(&tm_c);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t sf_col0 = kAccCols;
  if (threadIdx.x == 0) pdl_allow_dependents();
  pdl_wait();
  TRACE_DECL;
  if (threadIdx.x == 0) TRACE_STAMP(9);
  TRACE_CLOCK(14);

  if (producer_index(warp) >= 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    // K tile g of the pair's sequence goes to producer g % kProducers, stage g % S.
    const int pidx = producer_index(warp);
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_of(p.b_evict);
      int g = 0;
      WorkIter wi(p, pair_id, npairs);
      int t, k0, k1;
      for (bool first = true; !abort_flag && wi.next(p, KT, t, k0, k1); first = false) {
        int mb, nb, l;
        tile_coords(p, t, mb, nb, l);
        const int arow = mb * 256 + static_cast<int>(rank) * 128;
        const int brow = kDual ? nb * 128 : nb * 256 + static_cast<int>(rank) * 128;
        const CUtensorMap* bmap = (kDual && rank) ? &tm_b2 : &tm_b;
        const uint8_t* sfa_src = p.sfa + l * p.sfa_lstride + static_cast<int64_t>(arow / 128) * p.K * 8;
        // SFB blocks 0 and 1 of the N=256 operand: B rows [0,128), [128,256)
        // of the tile (dual: the B1 and the B2 tile).
        const uint8_t* sfb_src0 = p.sfb + l * p.sfb_lstride + static_cast<int64_t>(kDual ? nb : 2 * nb) * p.K * 8;
        const uint8_t* sfb_src1 = kDual ? p.sfb2 + l * p.sfb2_lstride + static_cast<int64_t>(nb) * p.K * 8
                                        : sfb_src0 + static_cast<int64_t>(p.K) * 8;
        for (int kt = k0; kt < k1; ++kt, ++g) {
          if (g % kProducers != pidx) continue;
          const int stage = g % S;
          const uint32_t phase = (g / S) & 1;
          if (!TRW(3, mbar_wait(&empty[stage], phase ^ 1))) {
            set_status(p.status, kStatusTimeoutEmpty);
            abort_flag = 1;
            break;
          }
          uint8_t* st = smem + stage * kStage;
          const uint32_t bar0 = map_peer(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], kTx);
          if (!(p.inject && blockIdx.x == 0 && first && kt == k0))
            tma_load_3d_pair(st, &tm_a, bar0, kt * kBKBytes, arow, l, pol_a);
          tma_load_3d_pair(st + kA, bmap, bar0, kt * kBKBytes, brow, l, pol_b);
          // Scales into this CTA's own shared memory, on its own barrier: SFA
          // of its 128 rows, SFB of both 128-row blocks of the tile's N.
          const uint32_t sf_bytes = sf_run_bytes(p.K, kt);
          mbar_arrive_expect_tx(&sf_full[stage], 3 * sf_bytes);
          bulk_load(st + kA + kB, sfa_src + kt * kSfStageBytes, sf_bytes, &sf_full[stage], pol_a);
          bulk_load(st + kA + kB + kSfa, sfb_src0 + kt * kSfStageBytes, sf_bytes, &sf_full[stage], pol_b);
          bulk_load(st + kA + kB + kSfa + kSfStageBytes, sfb_src1 + kt * kSfStageBytes, sf_bytes, &sf_full[stage],
                    pol_b);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_nvf4(256, 256);
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      WorkIter wi(p, pair_id, npairs);
      int t, k0, k1;
      while (!abort_flag && ok && wi.next(p, KT, t, k0, k1)) {
        if (!TRW(16, mbar_wait(acc_empty, acc_phase ^ 1))) {
          set_status(p.status, kStatusTimeoutAccEmpty);
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        for (int kt = k0; kt < k1; ++kt) {
          if (!TRW(0, mbar_wait_cluster(&full[stage], phase))) {
            set_status(p.status, kStatusTimeoutFull);
            abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          TRACE_ISSUE_BEGIN;
          const uint32_t st = smem_u32(smem + stage * kStage);
          const uint32_t sfc = tmem_base + sf_col0 + stage * kSfCols;
          const int nkk = ksteps(p.K, kt);
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk)
            if (kk < nkk)
              mma_nvf4_pair(tmem_base, desc_kmajor_sw128(st + kk * (kMmaK / 2)),
                          desc_kmajor_sw128(st + kA + kk * (kMmaK / 2)), idesc, sfc + 4 * kk, sfc + 16 + 8 * kk,
                          (kt != k0 || kk != 0) ? 1u : 0u);
          tc_commit_pair_mc(&empty[stage], 0x3);
          TRACE_ISSUE_END;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair_mc(acc_full, 0x3);
        TRACE_STAMP(10);
#ifdef NVFP4_TRACE
        if (trace[18] == 0) trace[18] = global_timer_ns(); else trace[19] = global_timer_ns();
#endif
        acc_phase ^= 1;
      }
      tc_commit_pair(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp >= 6 && warp <= 9) {
    // ------------------------------------------------------------ scale writers (both CTAs)
    // Warps 6..9 of each CTA, one per TMEM lane quarter, write the CTA's own
    // scale runs into its own TMEM with tcgen05.st, in the layout
    // tcgen05.cp.32x128b.warpx4 would leave (SFA step kk at column 4*kk; SFB
    // block j of step kk at 16 + 4*(2*kk + j)), then arrive on the leader's
    // full[stage], which the leader's MMA thread waits for.
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t ready0 = map_peer(smem_u32(full), 0);
    int stage = 0;
    uint32_t phase = 0;
    int total = 0;
    {
      WorkIter wi(p, pair_id, npairs);
      int t, k0, k1;
      while (wi.next(p, KT, t, k0, k1)) total += k1 - k0;
    }
    for (int i = 0; i < total; ++i) {
      const bool got = TRW(4, mbar_wait(&sf_full[stage], phase));
      if (!__all_sync(0xffffffffu, got && !abort_flag)) {
        if (lane == 0 && !got) set_status(p.status, kStatusTimeoutFull);
        abort_flag = 1;
        break;
      }
      const uint8_t* sf = smem + stage * kStage + kA + kB + lane * 16;
      const uint32_t sfc = tmem_base + lane_base + sf_col0 + stage * kSfCols;
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint4 v = *reinterpret_cast<const uint4*>(sf + r * kSfStageBytes + kk * kSfBlockBytes);
          tmem_st_32x32b_x4(sfc + (r == 0 ? 4 * kk : 16 + 4 * (2 * kk + (r - 1))), v);
        }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      // The stores are complete (tcgen05.wait::st) and ordered before this
      // signal (tcgen05.fence::before_thread_sync), so a relaxed arrive is
      // enough; a release arrive at cluster scope per stage measured ~1500
      // cycles and made this signal the pair kernel's bottleneck.
      if (lane == 0) mbar_arrive_cluster_relaxed(ready0 + stage * 8);
      if (++stage == S) {
        stage = 0;
        phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const uint32_t acc_empty0 = map_peer(smem_u32(acc_empty), 0);
    uint32_t acc_phase = 0;
    WorkIter wi(p, pair_id, npairs);
    int t, k0, k1;
    // Stream-K slots and flags are per CTA: worker (pair) w, rank r -> 2w + r.
    const int my_slot = pair_id * 2 + static_cast<int>(rank);
    while (wi.next(p, KT, t, k0, k1)) {
      int mb, nb, l;
      tile_coords(p, t, mb, nb, l);
      // All four epilogue warps agree (named barrier 1) before any of them
      // goes on, so none is ever left alone at a named barrier below.
      if (!epi_all(TRW(6, mbar_wait(acc_full, acc_phase)))) {
        if (threadIdx.x == 64) set_status(p.status, kStatusTimeoutAccFull);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int rloc = q * 32 + lane;
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      // Every epilogue writes its results into the staging buffer in shared
      // memory, releases the accumulator as soon as TMEM has been read, and
      // one thread (64) stores the buffer with TMA / bulk copies while the
      // next item's MMAs run.  Before writing the buffer, the previous
      // item's stores must have finished reading it.
      auto stage_wait = [&]() {
        if (threadIdx.x == 64) bulk_wait_group_read0();
        epi_bar();
      };
      constexpr int kChunks = kDual ? 4 : 8;  // 32-column chunks of this CTA's output rows
      // fp16 output chunk o (32 columns = 64 bytes = four 16-byte units of
      // the row in box o / 2, units 4 * (o % 2) .. +3, at unit u ^ (row % 8)).
      auto stage_half = [&](int o, const uint32_t (&r)[32]) {
        uint8_t* box = outbuf + (o >> 1) * kOutBox + rloc * 128;
        const int sw = rloc & 7;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 v;
          __half2 h0 = __floats2half2_rn(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
          __half2 h1 = __floats2half2_rn(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
          __half2 h2 = __floats2half2_rn(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
          __half2 h3 = __floats2half2_rn(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
          v.x = *reinterpret_cast<uint32_t*>(&h0);
          v.y = *reinterpret_cast<uint32_t*>(&h1);
          v.z = *reinterpret_cast<uint32_t*>(&h2);
          v.w = *reinterpret_cast<uint32_t*>(&h3);
          const int u = 4 * (o & 1) + j;
          *reinterpret_cast<uint4*>(box + ((u ^ sw) << 4)) = v;
        }
      };
      // Release the accumulator and store the staged fp16 tile to C.
      auto release_and_store_c = [&]() {
        tc_fence_before();
        mbar_arrive_cluster_relaxed(acc_empty0);
        fence_proxy_async_smem();
        epi_bar();
        if (threadIdx.x == 64) {
          const int y = mb * 256 + static_cast<int>(rank) * 128;
          const int x = nb * (kDual ? 128 : 256) * 2;  // bytes
#pragma unroll
          for (int bx = 0; bx < kChunks / 2; ++bx) tma_store_3d(&tm_c, outbuf + bx * kOutBox, x + bx * 128, y, l);
          bulk_commit_group();
        }
      };
      if (!p.streamk) {
        // Whole tile (the common case).
        stage_wait();
#pragma unroll 1
        for (int o = 0; o < kChunks; ++o) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tacc + o * 32, r);
          if (kDual) {
            uint32_t r2[32];
            tmem_ld_32x32b_x32(tacc + o * 32 + 128, r2);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              r[i] = __float_as_uint(silu_mul(__uint_as_float(r[i]), __uint_as_float(r2[i])));
          } else {
            tmem_wait_ld();
          }
          stage_half(o, r);
        }
        release_and_store_c();
      } else if (k0 > 0) {
        // Contributor: this CTA's 128 rows of the partial tile (fp32) to its
        // slot, laid out [column group][float4 index][row][4 floats] (16 KB
        // per 32-column group), staged in shared memory in that layout and
        // written by bulk stores four groups (64 KB) at a time; then its flag.
        float* slot_base = p.sk_partial + static_cast<int64_t>(my_slot) * (128 * 256);
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          stage_wait();
          float4* stg = reinterpret_cast<float4*>(outbuf) + rloc;
#pragma unroll 1
          for (int gi = 0; gi < 4; ++gi) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tacc + (4 * h + gi) * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i)
              stg[(gi * 8 + i) * 128] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                                    __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
          }
          if (h == 1) {
            tc_fence_before();
            mbar_arrive_cluster_relaxed(acc_empty0);
          }
          fence_proxy_async_smem();
          epi_bar();
          if (threadIdx.x == 64) {
            bulk_store(slot_base + h * (128 * 128), outbuf, 128 * 128 * 4);
            bulk_commit_group();
          }
        }
        if (threadIdx.x == 64) {
          bulk_wait_group0();  // the partial is in global memory
          fence_proxy_async_all();
          __threadfence();
          st_release_gpu(p.sk_flag + my_slot, 1);
#ifdef NVFP4_TRACE
          g_gemm_trace[blockIdx.x * 32 + 22] = global_timer_ns();
#endif
        }
      } else {
        // Whole tile, or the finaliser of a tile whose K tiles [k1, KT)
        // the following pairs [pair_id + 1, c_end) computed.
        int c_end = pair_id + 1;
        if (k1 < KT) {
          const int64_t tile_end = sk_tile_end(p, t, KT);
          while (c_end < npairs && sk_begin(p, c_end, npairs) < tile_end) ++c_end;
          bool ok = true;
          if (threadIdx.x == 64) {
            for (int c = pair_id + 1; c < c_end && ok; ++c)
              if (sk_has_range(p, c, npairs)) ok = flag_wait(p.sk_flag + 2 * c + rank);
            if (ok)
              for (int c = pair_id + 1; c < c_end; ++c) p.sk_flag[2 * c + rank] = 0;  // ready for the next launch
            else
              set_status(p.status, kStatusTimeoutPeer);
            fence_proxy_async_all();
#ifdef NVFP4_TRACE
            g_gemm_trace[blockIdx.x * 32 + 20] = global_timer_ns();
#endif
          }
          if (!epi_all(ok)) {
            abort_flag = 1;
            break;
          }
        }
        // The contributors' partials are streamed into shared memory (free
        // now: this is the CTA's last segment and its MMAs are complete) by
        // bulk copies of 16 KB chunks, one (contributor, 32-column group)
        // each, through a ring of kFixBufs buffers; plain loads of the same
        // data from L2 were latency-bound (~17 GB/s per SM).
        int contrib[kMaxContrib];
        int nc = 0;
        for (int c = pair_id + 1; c < c_end; ++c)
          if (sk_has_range(p, c, npairs) && nc < kMaxContrib) contrib[nc++] = c;
        constexpr int kHalves = kDual ? 2 : 1;  // accumulator groups per output chunk
        const int nchunks = kChunks * kHalves * nc;
        auto issue = [&](int q) {  // chunk q -> ring buffer q % kFixBufs
          const int j = q % nc, h = (q / nc) % kHalves, o = q / (nc * kHalves);
          const int g = o + h * 4;
          const uint8_t* src = reinterpret_cast<const uint8_t*>(p.sk_partial) +
                               (static_cast<int64_t>(2 * contrib[j] + rank) * 8 + g) * kFixChunk;
          mbar_arrive_expect_tx(&fix_full[q % kFixBufs], kFixChunk);
          bulk_load(smem + (q % kFixBufs) * kFixChunk, src, kFixChunk, &fix_full[q % kFixBufs],
                    policy_evict_first());
        };
        stage_wait();
        bool fix_ok = true;
        if (!kDual) {
          // One contributor at a time: its whole partial (eight contiguous
          // 16 KB column groups) in one bulk copy, added into the
          // accumulator in TMEM (tcgen05.ld, add, tcgen05.st) -- or, for the
          // last contributor, staged as fp16 for C.  Contributors are added
          // in pair order, the same order on every call.  (A ring of 16 KB
          // copies waited one by one cost ~0.7 us per chunk.)
          if (nc == 0) {
#pragma unroll 1
            for (int o = 0; o < kChunks; ++o) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(tacc + o * 32, r);
              tmem_wait_ld();
              stage_half(o, r);
            }
          }
#pragma unroll 1
          for (int j = 0; j < nc; ++j) {
            if (threadIdx.x == 64) {
              mbar_arrive_expect_tx(&fix_full[j % kFixBufs], 8 * kFixChunk);
              bulk_load(smem,
                        reinterpret_cast<const uint8_t*>(p.sk_partial) +
                            static_cast<int64_t>(2 * contrib[j] + rank) * 8 * kFixChunk,
                        8 * kFixChunk, &fix_full[j % kFixBufs], policy_evict_first());
            }
            fix_ok &= mbar_wait(&fix_full[j % kFixBufs], (j / kFixBufs) & 1);
#ifdef NVFP4_TRACE
            if (threadIdx.x == 64 && j == 0) g_gemm_trace[blockIdx.x * 32 + 23] = global_timer_ns();
#endif
            const bool last_c = j == nc - 1;
#pragma unroll 1
            for (int o = 0; o < kChunks; ++o) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(tacc + o * 32, r);
              const float4* buf = reinterpret_cast<const float4*>(smem + o * kFixChunk) + rloc;
              float4 v[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) v[i] = buf[i * 128];
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                r[4 * i] = __float_as_uint(__uint_as_float(r[4 * i]) + v[i].x);
                r[4 * i + 1] = __float_as_uint(__uint_as_float(r[4 * i + 1]) + v[i].y);
                r[4 * i + 2] = __float_as_uint(__uint_as_float(r[4 * i + 2]) + v[i].z);
                r[4 * i + 3] = __float_as_uint(__uint_as_float(r[4 * i + 3]) + v[i].w);
              }
              if (last_c)
                stage_half(o, r);
              else
                tmem_st_32x32b_x32(tacc + o * 32, r);
            }
            if (!last_c) {
              // Partial sums back in TMEM, and every thread done reading the
              // buffer before the next contributor's copy overwrites it.
              tmem_wait_st();
              fence_proxy_async_smem();
              epi_bar();
            }
          }
#ifdef NVFP4_TRACE
          if (threadIdx.x == 64) g_gemm_trace[blockIdx.x * 32 + 24] = global_timer_ns();
#endif
        } else {
          // Dual GEMM: both accumulator halves per output chunk, streamed as
          // 16 KB chunks (one per contributor and 32-column group) through
          // a ring of kFixBufs buffers.
          if (threadIdx.x == 64)
            for (int q = 0; q < nchunks && q < kFixBufs; ++q) issue(q);
          int q = 0;
#pragma unroll 1
          for (int o = 0; o < kChunks; ++o) {
            uint32_t r[kHalves][32];
#pragma unroll
            for (int h = 0; h < kHalves; ++h) {
              tmem_ld_32x32b_x32(tacc + o * 32 + h * 128, r[h]);
              tmem_wait_ld();
              for (int j = 0; j < nc; ++j, ++q) {
                fix_ok &= mbar_wait(&fix_full[q % kFixBufs], (q / kFixBufs) & 1);
                const float4* buf = reinterpret_cast<const float4*>(smem + (q % kFixBufs) * kFixChunk) + rloc;
                float4 v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = buf[i * 128];
                if (nchunks > kFixBufs) {
                  // every thread has read buffer q: refill it with chunk q + kFixBufs
                  epi_bar();
                  if (threadIdx.x == 64 && q + kFixBufs < nchunks) {
                    fence_proxy_async_smem();
                    issue(q + kFixBufs);
                  }
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  r[h][4 * i] = __float_as_uint(__uint_as_float(r[h][4 * i]) + v[i].x);
                  r[h][4 * i + 1] = __float_as_uint(__uint_as_float(r[h][4 * i + 1]) + v[i].y);
                  r[h][4 * i + 2] = __float_as_uint(__uint_as_float(r[h][4 * i + 2]) + v[i].z);
                  r[h][4 * i + 3] = __float_as_uint(__uint_as_float(r[h][4 * i + 3]) + v[i].w);
                }
              }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i)
              r[0][i] = __float_as_uint(silu_mul(__uint_as_float(r[0][i]), __uint_as_float(r[kHalves - 1][i])));
            stage_half(o, r[0]);
          }
        }
        if (!fix_ok) set_status(p.status, kStatusTimeoutPeer);
        release_and_store_c();
#ifdef NVFP4_TRACE
        if (threadIdx.x == 64) g_gemm_trace[blockIdx.x * 32 + 21] = global_timer_ns();
#endif
      }
      acc_phase ^= 1;
    }
  }

#ifdef NVFP4_TRACE
  if (threadIdx.x == 64) TRACE_STAMP(11);
  if (warp == 1) TRACE_TOTAL(2);
  if (warp == 6) TRACE_TOTAL(5);
  if (warp == 2) TRACE_TOTAL(7);
  if (warp <= 2 || warp == 6) TRACE_FLUSH();
#endif
  // TMA stores of C issued by this CTA must be complete before it exits.
  if (threadIdx.x == 64) bulk_wait_group0();
  // The leader's MMAs read both CTAs' shared memory and write both TMEMs:
  // neither CTA frees TMEM or exits before the pair's work has drained.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) TRACE_STAMP(12);
  TRACE_CLOCK(15);
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 3-D byte tensor (inner bytes, rows, L) with a (box_inner x box_rows) box and
// 128-byte swizzle; rows past `rows` read as zero.
// Encoded tensor maps are cached (direct-mapped on the full argument tuple):
// encoding costs microseconds of host time per map, and callers typically
// reuse the same buffers call after call.
namespace {
struct TmaKey {
  const void* base;
  int rank;
  uint64_t dims[5], strides[4];
  uint32_t box[5];
  bool operator==(const TmaKey& o) const {
    if (base != o.base || rank != o.rank) return false;
    for (int i = 0; i < 5; ++i)
      if (dims[i] != o.dims[i] || box[i] != o.box[i]) return false;
    for (int i = 0; i < 4; ++i)
      if (strides[i] != o.strides[i]) return false;
    return true;
  }
};
struct TmaEntry {
  TmaKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kTmaCacheSize = 1024;
TmaEntry g_tma_cache[kTmaCacheSize];
std::mutex g_tma_mutex;

size_t tma_hash(const TmaKey& k) {
  uint64_t h = reinterpret_cast<uint64_t>(k.base) * 0x9E3779B97F4A7C15ull + k.rank;
  for (int i = 0; i < 5; ++i) h = (h ^ k.dims[i] ^ (uint64_t(k.box[i]) << 40)) * 0xBF58476D1CE4E5B9ull;
  for (int i = 0; i < 4; ++i) h = (h ^ k.strides[i]) * 0x94D049BB133111EBull;
  return static_cast<size_t>(h >> 40) % kTmaCacheSize;
}
}  // namespace

// Byte tensor of rank 3..5 (dims[0] innermost, strides in bytes for dims
// 1..rank-1) with a box of `box` and 128-byte swizzle; out-of-range rows read
// as zero.  Encoded maps are cached (direct-mapped on the full argument set):
// encoding costs microseconds of host time, and callers reuse buffers.
bool make_tma_u8(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                 const uint32_t* box) {
  TmaKey key{};
  key.base = base;
  key.rank = rank;
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i > 0) key.strides[i - 1] = strides[i - 1];
  }
  const size_t slot = tma_hash(key);
  {
    std::lock_guard<std::mutex> lock(g_tma_mutex);
    if (g_tma_cache[slot].valid && g_tma_cache[slot].key == key) {
      *map = g_tma_cache[slot].map;
      return true;
    }
  }
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    if (i > 0) st[i - 1] = strides[i - 1];
  }
  // Scale-factor maps (inner box of 256 bytes) are plain copies; operand maps
  // use the 128-byte swizzle tcgen05 descriptors expect.
  const CUtensorMapSwizzle swz = box[0] == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void*>(base), d, st, bx, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(g_tma_mutex);
  g_tma_cache[slot].key = key;
  g_tma_cache[slot].map = *map;
  g_tma_cache[slot].valid = true;
  return true;
}

bool make_tma_3d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t L,
                    uint64_t row_stride, uint64_t lstride, uint32_t box_inner, uint32_t box_rows) {
  const uint64_t dims[3] = {inner, rows, L};
  const uint64_t strides[2] = {row_stride, lstride};
  const uint32_t box[3] = {box_inner, box_rows, 1};
  return make_tma_u8(map, base, 3, dims, strides, box);
}

static bool make_operand_map(CUtensorMap* map, const void* base, int K2, int rows, int L, int64_t lstride,
                             int box_rows) {
  return make_tma_3d_u8(map, base, K2, rows, L, K2, lstride, kBKBytes, box_rows);
}

template <int BN, bool kDual>
static cudaError_t launch_impl(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  using Cfg = GemmConfig<BN, kDual>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN, kDual>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  CUtensorMap ta, tb, tb2, tc;
  const int K2 = g.K / 2;
  // C as bytes for the split-K epilogue: boxes of 128 rows x 64 bytes (32 columns), no swizzle.
  if (!make_operand_map(&ta, g.a, K2, g.M, g.L, g.a_lstride, kBM) ||
      !make_operand_map(&tb, g.b, K2, g.N, g.L, g.b_lstride, BN) ||
      (kDual && !make_operand_map(&tb2, g.b2, K2, g.N, g.L, g.b2_lstride, BN)) ||
      !make_tma_3d_u8(&tc, g.c, static_cast<uint64_t>(g.N) * 2, g.M, g.L, static_cast<uint64_t>(g.ldc) * 2,
                      static_cast<uint64_t>(g.c_lstride) * 2, 64, kBM)) {
    *why = "cuTensorMapEncodeTiled failed";
    return cudaErrorInvalidValue;
  }
  if (!kDual) tb2 = tb;
  GemmParams p;
  p.sfa = static_cast<const uint8_t*>(g.sfa);
  p.sfb = static_cast<const uint8_t*>(g.sfb);
  p.sfb2 = static_cast<const uint8_t*>(g.sfb2);
  p.c = static_cast<__half*>(g.c);
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.L = g.L;
  p.sfa_lstride = g.sfa_lstride;
  p.sfb_lstride = g.sfb_lstride;
  p.sfb2_lstride = g.sfb2_lstride;
  p.ldc = g.ldc;
  p.c_lstride = g.c_lstride;
  p.tiles_m = g.M / kBM;
  p.tiles_n = g.N / BN;
  p.num_tiles = p.tiles_m * p.tiles_n * g.L;
  p.group_m = p.tiles_m < 16 ? p.tiles_m : 16;
  p.status = g.status;
  p.splits = g.splits > 1 ? g.splits : 1;
  p.num_items = p.num_tiles * p.splits;
  p.streamk = (!kDual && p.splits == 1 && g.streamk && g.workspace) ? 1 : 0;
  p.sk_flag = static_cast<int*>(g.workspace);
  p.sk_partial = p.streamk ? reinterpret_cast<float*>(static_cast<uint8_t*>(g.workspace) + kStreamKFlagBytes) : nullptr;
  // Test hook for the bounded-wait path (tests/test_failure_detection.py):
  // the kernel then reports a pipeline timeout instead of hanging.  With
  // split K the other CTAs of CTA 0's cluster finish their main loops and
  // wait at the cluster barrier until CTA 0's bounded waits have run out.
  p.inject = g.inject ? 1 : 0;
  p.prefetch = g.prefetch;
  p.b_evict = g.b_evict;
  // Without split: a persistent grid.  With split K: one CTA per (tile,
  // split), the splits of a tile in one cluster.
  const int grid = p.splits == 1 ? (p.num_items < num_sms ? p.num_items : num_sms) : p.num_items;
  p.dp_tiles = g.streamk_pure ? 0 : (p.num_tiles / grid) * grid;
  p.units = static_cast<int64_t>(p.num_tiles - p.dp_tiles) * ((g.K + kBK - 1) / kBK);
  if (p.streamk && grid * (kBM * BN * 4) + kStreamKFlagBytes > static_cast<int64_t>(g.workspace_bytes)) {
    *why = "stream-K workspace too small";
    return cudaErrorInvalidValue;
  }
  return launch_pdl(gemm_kernel<BN, kDual>, dim3(grid), dim3(kThreads), Cfg::kSmemBytes, stream, p.splits, ta, tb,
                    tb2, tc, p);
}

// Tile width and K splits for a problem.  Problems with fewer tiles than SMs
// (the dual GEMM's M=256 shapes, M=128 GEMMs) split K so more SMs work; the
// splits of a tile form one thread-block cluster and are reduced on chip.
// NVFP4_GEMM_BN / NVFP4_SPLITS override the choice (tuning only).
// Clusters of `S` CTAs of this kernel that can be resident at once (clusters
// must fit inside one GPC, so with ~220 KB of shared memory per CTA this is
// less than num_sms / S for S = 3, 5, 6, 7, 8).  Cached per device.
template <int BN, bool kDual>
static int max_active_clusters(int S) {
  using Cfg = GemmConfig<BN, kDual>;
  static int cache[16][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16 || S < 1 || S > 8) return 0;
  if (!cache[dev][S]) {
    if (cudaFuncSetAttribute(gemm_kernel<BN, kDual>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) !=
        cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S * 64);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = S;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<BN, kDual>, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = -1;  // unknown: fall back to num_sms / S
    }
    cache[dev][S] = n;
  }
  return cache[dev][S];
}

GemmPlan gemm_plan(int M, int N, int K, int L, bool dual, int num_sms, const EnvOptions& opt) {
  GemmPlan pl;
  const int forced_bn = opt.gemm_bn;
  pl.bn = (!dual && N % 256 == 0 && forced_bn != 128) ? 256 : 128;
  const int tiles = (M / 128) * (N / pl.bn) * L;
  const int KT = (K + 255) / 256;
  const int ngroups = pl.bn / 32;  // a split owns at least one 32-column group of the tile
  int splits = 1;
  if (tiles < num_sms) splits = num_sms / tiles;
  {
    // Each extra split rank adds ~1 us of DSMEM exchange; each K tile a CTA
    // runs costs ~0.36 us (same-box measurements on the M=128 / M=256
    // shapes), so the time a + (S-1) + 0.36*KT/S is least near S = sqrt(0.36*KT):
    // 2 for K=2048, 3 for K=7168, 5 for K=16384.  Measured: 128x7168x2048
    // 12.9 -> 10.9 us, 128x4096x7168 17.1 -> 15.2 us against filling the SMs.
    int model = static_cast<int>(lrint(sqrt(0.36 * KT)));
    if (model < 1) model = 1;
    if (splits > model) splits = model;
  }
  const int forced = opt.splits;
  if (forced > 0) splits = forced;
  if (splits > KT / 2) splits = KT / 2;  // at least two K tiles per split
  if (splits > ngroups) splits = ngroups;
  if (splits > 8) splits = 8;            // portable cluster size
  if (tiles * splits > num_sms) splits = num_sms / tiles;
  // All clusters must be resident in one wave: a cluster that starts late
  // holds up its whole tile.
  while (splits > 1) {
    int fit = dual ? max_active_clusters<128, true>(splits)
                   : (pl.bn == 256 ? max_active_clusters<256, false>(splits) : max_active_clusters<128, false>(splits));
    if (fit < 0) fit = num_sms / splits;
    if (tiles <= fit) break;
    --splits;
  }
  // The split-K exchange reuses the pipeline stages for the receive slots
  // and, after them, the staged output share: both must fit.
  while (splits > 1) {
    const int ng = pl.bn / 32, share = (ng + splits - 1) / splits;
    const int gf = 32 * (dual ? 2 : 1);
    const size_t recv = static_cast<size_t>(splits - 1) * share * (gf / 4) * kBM * 16;
    const size_t need = ((recv + 1023) & ~static_cast<size_t>(1023)) + static_cast<size_t>(share) * kBM * 64;
    const size_t have = dual ? static_cast<size_t>(GemmConfig<128, true>::kStages) * GemmConfig<128, true>::kStageBytes
                        : pl.bn == 256 ? static_cast<size_t>(GemmConfig<256, false>::kStages) * GemmConfig<256, false>::kStageBytes
                                       : static_cast<size_t>(GemmConfig<128, false>::kStages) * GemmConfig<128, false>::kStageBytes;
    if (need <= have) break;
    --splits;
  }
  pl.splits = splits < 1 ? 1 : splits;
  pl.workspace_bytes = 0;
  pl.b_evict = 0;
  pl.streamk = 0;
  pl.streamk_pure = 0;
  pl.pair = 0;
  // 2-CTA pairs (256x256 tiles) whenever the shape allows: per K tile each
  // SM moves 32 KB through shared memory for TMA writes and 32 KB for MMA
  // reads instead of 48 + 48 KB with 128x256 tiles (measured +17% on
  // 1024x7168x16384, +27% on 16384^3).  NVFP4_PAIR=0 keeps 1-CTA tiles.
  // The dual GEMM runs on pairs (256 x (128 B1 + 128 B2) tiles, whole tiles)
  // when M % 256 == 0 and the pair tiles fill at least ~2/3 of the pairs
  // (measured: 512x4096x7168 18.8 us against 20.4 on 1-CTA tiles with K
  // split in clusters; with half the pairs busy, 256x4096x7168, the 1-CTA
  // split is faster).  Splitting K across pairs (stream-K, NVFP4_STREAMK=2)
  // costs a trip of fp32 partial tiles through L2, measured slower.
  const bool pair_on = opt.pair == 1, pair_off = opt.pair == 0;
  pl.pair = (!dual && pl.bn == 256 && pl.splits == 1 && M % 256 == 0 && !pair_off) ? 1 : 0;
  if (dual && M % 256 == 0 && !pair_off && (pair_on || 3 * ((M / 256) * (N / 128) * L) >= 2 * (num_sms / 2))) {
    pl.pair = 1;
    pl.splits = 1;
  }
  // Stream-K (hybrid) when whole tiles leave the last wave part-empty: e.g.
  // 112 pair tiles on 74 pairs run as two tile-waves, 38 pairs busy in the
  // second; instead every worker takes one whole tile and then ~0.51 of a
  // tile's K range of the 38 left over.  Used when the busiest worker's K
  // tiles drop by more than 10%.  NVFP4_STREAMK: 1 force on, 2 force the
  // pure form (no whole-tile waves), -1 force off.
  const int forced_sk = opt.streamk;
  const int wtiles = pl.pair ? (M / 256) * (N / (dual ? 128 : 256)) * L : tiles;
  const int workers = pl.pair ? num_sms / 2 : num_sms;
  if (pl.pair && wtiles < workers && forced_sk == 2) {
    // Fewer pair tiles than pairs: pure stream-K spreads the K tiles over all
    // pairs (a tile's K range then spans about workers / tiles pairs).
    pl.streamk = 1;
    pl.streamk_pure = 1;
    pl.workspace_bytes = kStreamKFlagBytes + static_cast<size_t>(2 * workers) * 128 * 256 * 4;
  } else if ((pl.pair || (!dual && pl.splits == 1)) && forced_sk >= 0 && wtiles > workers) {
    const int64_t classic = static_cast<int64_t>((wtiles + workers - 1) / workers) * KT;
    const int rest = wtiles % workers;
    const int64_t hybrid =
        static_cast<int64_t>(wtiles / workers) * KT + (static_cast<int64_t>(rest) * KT + workers - 1) / workers + 2;
    if (forced_sk >= 1 || (rest != 0 && hybrid * 10 < classic * 9)) {
      pl.streamk = 1;
      pl.streamk_pure = forced_sk == 2 ? 1 : 0;
      pl.workspace_bytes =
          kStreamKFlagBytes + static_cast<size_t>(pl.pair ? 2 * workers : workers) * 128 * 256 * 4;
    }
  }
  return pl;
}

template <bool kDual>
static cudaError_t launch_pair(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  static bool attr_done[64] = {false};
  static int max_pairs[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<kDual>, cudaFuncAttributeMaxDynamicSharedMemorySize, pair::kSmem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kPairThreads);
    cfg.dynamicSmemBytes = pair::kSmem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<kDual>, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = num_sms / 2;
    }
    max_pairs[dev] = n;
    attr_done[dev] = true;
  }
  const uint64_t K2 = g.K / 2;
  CUtensorMap ta, tb, tb2, tc;
  // C as bytes: rows of N * 2 bytes at a stride of ldc * 2, boxes of 128 rows x 128 bytes.
  if (!make_operand_map(&ta, g.a, K2, g.M, g.L, g.a_lstride, 128) ||
      !make_operand_map(&tb, g.b, K2, g.N, g.L, g.b_lstride, 128) ||
      (kDual && !make_operand_map(&tb2, g.b2, K2, g.N, g.L, g.b2_lstride, 128)) ||
      !make_tma_3d_u8(&tc, g.c, static_cast<uint64_t>(g.N) * 2, g.M, g.L, static_cast<uint64_t>(g.ldc) * 2,
                      static_cast<uint64_t>(g.c_lstride) * 2, 128, 128)) {
    *why = "cuTensorMapEncodeTiled failed";
    return cudaErrorInvalidValue;
  }
  GemmParams p{};
  p.sfa = static_cast<const uint8_t*>(g.sfa);
  p.sfb = static_cast<const uint8_t*>(g.sfb);
  p.sfb2 = static_cast<const uint8_t*>(g.sfb2);
  p.sfa_lstride = g.sfa_lstride;
  p.sfb_lstride = g.sfb_lstride;
  p.sfb2_lstride = g.sfb2_lstride;
  p.c = static_cast<__half*>(g.c);
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.L = g.L;
  p.ldc = g.ldc;
  p.c_lstride = g.c_lstride;
  p.tiles_m = g.M / 256;
  p.tiles_n = g.N / (kDual ? 128 : 256);
  p.num_tiles = p.tiles_m * p.tiles_n * g.L;
  // Raster: groups of 16 256-row blocks sweep N (16384^3: DRAM reads 2.73 ->
  // 2.00 GB per launch against groups of 8, one ncu pass each).
  p.group_m = p.tiles_m < 16 ? p.tiles_m : 16;
  p.status = g.status;
  p.inject = g.inject ? 1 : 0;
  p.b_evict = g.b_evict;
  p.splits = 1;
  p.num_items = p.num_tiles;
  p.streamk = (g.streamk && g.workspace) ? 1 : 0;
  // Whole tiles: at most one pair per tile.  Stream-K: every co-resident
  // pair (at most one per K tile).
  int pairs = max_pairs[dev < 64 ? dev : 0];
  // (Stream-K: at most 8 pairs per tile, so a tile's K range spans at most
  // ~10 pairs, within the finaliser's pair::kMaxContrib.)
  const int64_t kts = (g.K + kBK - 1) / kBK;
  const int64_t work = p.streamk ? static_cast<int64_t>(p.num_tiles) * (kts < 8 ? kts : 8) : p.num_tiles;
  if (pairs > work) pairs = static_cast<int>(work);
  if (pairs < 1) pairs = 1;
  p.dp_tiles = g.streamk_pure ? 0 : (p.num_tiles / pairs) * pairs;
  p.units = static_cast<int64_t>(p.num_tiles - p.dp_tiles) * ((g.K + kBK - 1) / kBK);
  p.sk_flag = static_cast<int*>(g.workspace);
  p.sk_partial = p.streamk ? reinterpret_cast<float*>(static_cast<uint8_t*>(g.workspace) + kStreamKFlagBytes) : nullptr;
  if (p.streamk && static_cast<size_t>(2 * pairs) * 128 * 256 * 4 + kStreamKFlagBytes > g.workspace_bytes) {
    *why = "stream-K workspace too small";
    return cudaErrorInvalidValue;
  }
  return launch_pdl(gemm_pair_kernel<kDual>, dim3(2 * pairs), dim3(kPairThreads), pair::kSmem, stream, 2, ta, tb,
                    kDual ? tb2 : tb, tc, p);
}

cudaError_t launch_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  if (g.pair) return launch_pair<false>(g, num_sms, stream, why);
  if (g.bn == 256) return launch_impl<256, false>(g, num_sms, stream, why);
  return launch_impl<128, false>(g, num_sms, stream, why);
}

cudaError_t launch_dual_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  if (g.pair) return launch_pair<true>(g, num_sms, stream, why);
  return launch_impl<128, true>(g, num_sms, stream, why);
}

}  // namespace nvfp4

#ifdef NVFP4_TRACE
extern "C" __attribute__((visibility("default"))) int nvfp4_dbg_gemm_trace(unsigned long long* host) {
  if (cudaMemcpyFromSymbol(host, nvfp4::g_gemm_trace, sizeof(nvfp4::g_gemm_trace)) != cudaSuccess) return 1;
  static unsigned long long zero[1024 * 32];
  return cudaMemcpyToSymbol(nvfp4::g_gemm_trace, zero, sizeof(zero)) != cudaSuccess;
}
#endif
