// NVFP4 GEMV fed by TMA, with the tensor core as the dot-product engine.
//
//   c[m, l] = fp16( sum_k (a[m,k,l] sfa[m,k/16,l]) (b[0,k,l] sfb[0,k/16,l]) )
//   semantics of ref_kernel, problems/nvidia/nvfp4_gemv/reference.py:28-54
//
// The GEMV is bound by HBM reads of A (K/2 + K/16 bytes per row).  A SIMT
// dot product needs about one instruction per element just to widen and
// multiply e2m1 pairs, which issue-limits it well below the HBM rate, so this
// kernel moves A with TMA straight into shared memory and lets
// tcgen05.mma kind::mxf4nvf4 (M=128, N=32, K=64) do the block-scaled
// multiply-accumulate in TMEM: B is b's row 0 in a 32-row tile whose other
// rows are TMA zero fill, and only column 0 of the accumulator is read.
//
// Work split: the (l, 128-row block, 256- or 512-wide K range) units are cut into one
// contiguous range per CTA (one CTA per SM), so every SM streams the same
// number of bytes.  A CTA accumulates each run of units of one row block in
// TMEM; a block whose K range is split over several CTAs is finished by the
// last contributor, which adds the partial sums in CTA order from a workspace
// (deterministic) and resets the block's arrival counter.
//
// Warp roles (7 warps): 0 TMA producer, 1 MMA issuer + TMEM owner,
// 2..5 epilogue, 6 scale copier (tcgen05.cp of the stage's scale blocks,
// issued apart from the MMAs so the two overlap).
#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {

namespace gemvtc {

constexpr int kBM = 128;
constexpr int kBN = 32;         // MMA N; only row 0 of B is real
constexpr int kBK = 256;        // K elements per sub-tile (128 bytes of a row)
constexpr int kBKBytes = kBK / 2;
constexpr int kASub = kBM * kBKBytes;  // 16 KB
constexpr int kBSub = kBN * kBKBytes;  // 4 KB
constexpr int kSfSub = 2048;           // one 128-row scale block for 4 MMA steps
constexpr int kAccCols = kBN;
constexpr int kAccBufs = 2;
constexpr int kTmemCols = 512;
constexpr int kThreads = 224;

// A unit is SUB consecutive 256-wide K sub-tiles of one 128-row block; one
// stage holds one unit and is filled by one TMA request per operand (a box
// of SUB 128-byte columns), so wider units mean fewer, larger requests.
template <int SUB>
struct Cfg {
  static constexpr int kStages = SUB == 1 ? 8 : 4;
  static constexpr int kA = SUB * kASub;
  static constexpr int kB = SUB * kBSub;
  static constexpr int kSf = SUB * kSfSub;
  static constexpr int kStageBytes = kA + kB + 2 * kSf;
  static constexpr int kSfCols = 32 * SUB;  // per stage: SFA 16 + SFB 16 per sub-tile
  static_assert(kAccBufs * kAccCols + kStages * kSfCols <= kTmemCols, "TMEM budget");
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;
};

}  // namespace gemvtc

struct GemvTcParams {
  const uint8_t* sfa;  // blocked scales of A, batch l at + l * sfa_lstride
  const uint8_t* sfb;  // blocked scales of b (row block 0 used)
  __half* c;
  float* ws;      // partial sums: [block][slot][128]
  int* counters;  // arrivals per block
  int M, K, L;
  int64_t sfa_lstride, sfb_lstride, c_lstride;
  int units, kt_per_block, blocks_per_l, slots;
  int* status;
  int inject;  // test hook: CTA 0 withholds its first A load
};

// First unit of CTA `c` when `units` are split over `ctas` CTAs.
__host__ __device__ __forceinline__ int unit_begin(int c, int units, int ctas) {
  return static_cast<int>((static_cast<int64_t>(c) * units) / ctas);
}
// CTA whose range holds unit `u` (largest c with unit_begin(c) <= u).
__host__ __device__ __forceinline__ int unit_owner(int u, int units, int ctas) {
  int c = static_cast<int>(((static_cast<int64_t>(u) + 1) * ctas - 1) / units);
  if (c >= ctas) c = ctas - 1;
  while (c > 0 && unit_begin(c, units, ctas) > u) --c;
  while (c + 1 < ctas && unit_begin(c + 1, units, ctas) <= u) ++c;
  return c;
}

__device__ __forceinline__ void tmem_ld_32x32b_x1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ int atom_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

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

template <int SUB>
__global__ void __launch_bounds__(gemvtc::kThreads, 1)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const GemvTcParams p) {
  using namespace gemvtc;
  using C = Cfg<SUB>;
  constexpr int kStages = C::kStages;
  constexpr int kStageBytes = C::kStageBytes;
  constexpr int kSfCols = C::kSfCols;
  constexpr int kTxBytes = kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* sf_ready = bars + 2 * kStages;
  uint64_t* acc_full = bars + 3 * kStages;
  uint64_t* acc_empty = acc_full + kAccBufs;
  uint64_t* drain = acc_empty + kAccBufs;  // [0] MMA thread, [1] scale copier
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  __shared__ volatile int abort_flag;
  __shared__ int last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = unit_begin(blockIdx.x, p.units, gridDim.x);
  const int u1 = unit_begin(blockIdx.x + 1, p.units, gridDim.x);
  const int KT = p.kt_per_block;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_ready[s], 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    fence_barrier_init();
    prefetch_tensormap(&tm_a);
    prefetch_tensormap(&tm_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t sf_col0 = kAccBufs * kAccCols;
  if (threadIdx.x == 0) pdl_allow_dependents();
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_stream = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      for (int u = u0; u < u1 && !abort_flag; ++u) {
        const int blk = u / KT, kt = u - blk * KT;
        const int l = blk / p.blocks_per_l, mb = blk - l * p.blocks_per_l;
        if (!mbar_wait(&empty[stage], phase ^ 1)) {
          if (p.status) atomicCAS(p.status, 0, kStatusTimeoutEmpty);
          abort_flag = 1;
          break;
        }
        uint8_t* st = smem + stage * kStageBytes;
        mbar_arrive_expect_tx(&full[stage], kTxBytes);
        if (!(p.inject && blockIdx.x == 0 && u == u0))
          tma_load_4d(st, &tm_a, &full[stage], 0, mb * kBM, kt * SUB, l, pol_stream);
        tma_load_4d(st + C::kA, &tm_b, &full[stage], 0, 0, kt * SUB, l, pol_keep);
        bulk_load(st + C::kA + C::kB,
                  p.sfa + l * p.sfa_lstride + static_cast<int64_t>(mb) * p.K * 8 + kt * C::kSf, C::kSf,
                  &full[stage], pol_stream);
        bulk_load(st + C::kA + C::kB + C::kSf, p.sfb + l * p.sfb_lstride + kt * C::kSf, C::kSf, &full[stage],
                  pol_keep);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------ scale copier
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int u = u0; u < u1 && !abort_flag; ++u) {
        if (!mbar_wait(&full[stage], phase)) {
          if (p.status) atomicCAS(p.status, 0, kStatusTimeoutFull);
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sf = smem_u32(smem + stage * kStageBytes + C::kA + C::kB);
        const uint32_t sfc = tmem_base + sf_col0 + stage * kSfCols;
#pragma unroll
        for (int j = 0; j < SUB; ++j)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            tmem_cp_32x128b_x4(sfc + 32 * j + 4 * kk, desc_sf_block(sf + j * kSfSub + kk * 512));
            tmem_cp_32x128b_x4(sfc + 32 * j + 16 + 4 * kk, desc_sf_block(sf + C::kSf + j * kSfSub + kk * 512));
          }
        tc_commit(&sf_ready[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      tc_commit(&drain[1]);
      mbar_wait(&drain[1], 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kBM, kBN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int u = u0; u < u1 && !abort_flag; ++u) {
        const int kt = u % KT;
        const bool seg_begin = (u == u0) || kt == 0;
        const bool seg_end = (u == u1 - 1) || kt == KT - 1;
        if (seg_begin) {
          if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) {
            if (p.status) atomicCAS(p.status, 0, kStatusTimeoutAccEmpty);
            abort_flag = 1;
            break;
          }
          tc_fence_after();
        }
        if (!mbar_wait(&full[stage], phase) || !mbar_wait(&sf_ready[stage], phase)) {
          if (p.status) atomicCAS(p.status, 0, kStatusTimeoutFull);
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + stage * kStageBytes);
        const uint32_t sfc = tmem_base + sf_col0 + stage * kSfCols;
        const uint32_t d = tmem_base + acc * kAccCols;
#pragma unroll
        for (int j = 0; j < SUB; ++j)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_nvf4(d, desc_kmajor_sw128(st + j * kASub + kk * 32), desc_kmajor_sw128(st + C::kA + j * kBSub + kk * 32),
                     idesc, sfc + 32 * j + 4 * kk, sfc + 32 * j + 16 + 4 * kk, (seg_begin && j == 0 && kk == 0) ? 0u : 1u);
        tc_commit(&empty[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
        if (seg_end) {
          tc_commit(&acc_full[acc]);
          if (++acc == kAccBufs) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
      tc_commit(&drain[0]);
      mbar_wait(&drain[0], 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;
    const int r = q * 32 + lane;  // row within the block == TMEM lane
    int acc = 0;
    uint32_t acc_phase = 0;
    int u = u0;
    while (u < u1) {
      const int blk = u / KT;
      const int seg_end_u = min(u1, (blk + 1) * KT);  // exclusive
      const bool whole = (u == blk * KT) && (seg_end_u == (blk + 1) * KT);
      // The four epilogue warps agree before any of them leaves, so none is
      // left waiting at a named barrier below.
      if (!epi_all(mbar_wait(&acc_full[acc], acc_phase))) {
        if (threadIdx.x == 64 && p.status) atomicCAS(p.status, 0, kStatusTimeoutAccFull);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      uint32_t v;
      tmem_ld_32x32b_x1(tmem_base + acc * kAccCols + (static_cast<uint32_t>(q * 32) << 16), v);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == kAccBufs) {
        acc = 0;
        acc_phase ^= 1;
      }
      const int l = blk / p.blocks_per_l, mb = blk - l * p.blocks_per_l;
      __half* crow = p.c + l * p.c_lstride + mb * kBM + r;
      const float x = __uint_as_float(v);
      if (whole) {
        *crow = __float2half_rn(x);
      } else {
        // Contributors of this block, in CTA order; our slot is our rank among them.
        const int first = unit_owner(blk * KT, p.units, gridDim.x);
        const int last = unit_owner((blk + 1) * KT - 1, p.units, gridDim.x);
        const int slot = blockIdx.x - first;
        float* wsb = p.ws + static_cast<int64_t>(blk) * p.slots * kBM;
        wsb[slot * kBM + r] = x;
        // The named barrier orders the 128 partial-sum stores before thread
        // 64's arrival, whose release (cumulative) publishes them; the last
        // arriver's acquire, passed on by the second barrier, orders its
        // CTA's reads after every contributor's stores.  (No full fences.)
        epi_bar();
        if (threadIdx.x == 64) last_flag = (atom_add_acq_rel_gpu(&p.counters[blk], 1) == last - first);
        epi_bar();
        if (last_flag) {
          float s = 0.f;
          for (int j = 0; j <= last - first; ++j) s += __ldcg(&wsb[j * kBM + r]);
          *crow = __float2half_rn(s);
          if (threadIdx.x == 64) p.counters[blk] = 0;
        }
        epi_bar();
      }
      u = seg_end_u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
bool make_tma_u8(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                 const uint32_t* box);

static int sub_of(int K) { return K % (2 * gemvtc::kBK) == 0 ? 2 : 1; }

static void plan(int M, int K, int L, int num_sms, int* units, int* grid, int* slots, int* blocks) {
  const int KT = K / (gemvtc::kBK * sub_of(K));
  *blocks = (M / gemvtc::kBM) * L;
  *units = *blocks * KT;
  *grid = *units < num_sms ? *units : num_sms;
  // Most CTAs whose unit ranges (each >= units/grid long) can meet one block.
  const int per_cta = *units / *grid;
  int s = per_cta > 0 ? (KT + per_cta - 1) / per_cta + 1 : KT;
  if (s > *grid) s = *grid;
  *slots = s;
}

// Workspace layout: a fixed region of kMaxCounterBlocks arrival counters
// (always at the start, so partial sums of one call never land on the
// counters of another), then the partial sums [block][slot][128].
size_t gemv_tc_workspace_bytes(int M, int K, int L, int num_sms) {
  int units, grid, slots, blocks;
  plan(M, K, L, num_sms, &units, &grid, &slots, &blocks);
  if (blocks > kGemvTcMaxCounterBlocks) return 0;
  return static_cast<size_t>(kGemvTcMaxCounterBlocks) * sizeof(int) +
         static_cast<size_t>(blocks) * slots * gemvtc::kBM * sizeof(float);
}

template <int SUB>
static cudaError_t launch_sub(const GemvTcArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  using namespace gemvtc;
  using C = Cfg<SUB>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<SUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  const uint64_t K2 = g.K / 2;
  // (128-byte column, row, 128-byte column index, batch) views of A and b;
  // b has one row, the MMA tile's other 31 rows read as zero.
  const uint64_t da[4] = {128, static_cast<uint64_t>(g.M), K2 / 128, static_cast<uint64_t>(g.L)};
  const uint64_t sa[3] = {K2, 128, static_cast<uint64_t>(g.a_lstride)};
  const uint32_t ba[4] = {128, kBM, SUB, 1};
  const uint64_t db[4] = {128, 1, K2 / 128, static_cast<uint64_t>(g.L)};
  const uint64_t sb[3] = {K2, 128, static_cast<uint64_t>(g.b_lstride)};
  const uint32_t bb[4] = {128, kBN, SUB, 1};
  CUtensorMap ta, tb;
  if (!make_tma_u8(&ta, g.a, 4, da, sa, ba) || !make_tma_u8(&tb, g.b, 4, db, sb, bb)) {
    *why = "cuTensorMapEncodeTiled failed";
    return cudaErrorInvalidValue;
  }
  int units, grid, slots, blocks;
  plan(g.M, g.K, g.L, num_sms, &units, &grid, &slots, &blocks);
  const size_t need = gemv_tc_workspace_bytes(g.M, g.K, g.L, num_sms);
  if (need == 0 || need > g.workspace_bytes) {
    *why = "workspace too small";
    return cudaErrorInvalidValue;
  }
  GemvTcParams p;
  p.sfa = static_cast<const uint8_t*>(g.sfa);
  p.sfb = static_cast<const uint8_t*>(g.sfb);
  p.c = static_cast<__half*>(g.c);
  p.M = g.M;
  p.K = g.K;
  p.L = g.L;
  p.sfa_lstride = g.sfa_lstride;
  p.sfb_lstride = g.sfb_lstride;
  p.c_lstride = g.c_lstride;
  p.kt_per_block = g.K / (kBK * SUB);
  p.blocks_per_l = g.M / kBM;
  p.units = units;
  p.slots = slots;
  p.counters = static_cast<int*>(g.workspace);
  p.ws = reinterpret_cast<float*>(p.counters + kGemvTcMaxCounterBlocks);
  p.status = g.status;
  p.inject = g.inject;
  return launch_pdl(gemv_tc_kernel<SUB>, dim3(grid), dim3(kThreads), C::kSmemBytes, stream, 1, ta, tb, p);
}

cudaError_t launch_gemv_tc(const GemvTcArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  if (sub_of(g.K) == 2) return launch_sub<2>(g, num_sms, stream, why);
  return launch_sub<1>(g, num_sms, stream, why);
}

}  // namespace nvfp4
