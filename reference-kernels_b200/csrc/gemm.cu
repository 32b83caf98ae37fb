// NVFP4 block-scaled GEMM and dual GEMM (fused SiLU gate) for sm_100a.
//
//   GEMM:  C[m,n,l] = fp16( sum_k (A sfA)[m,k,l] (B sfB)[n,k,l] )
//          ref_kernel of problems/nvidia/nvfp4_gemm/reference.py:27-53
//   Dual:  C[m,n,l] = fp16( silu(A.B1^T) * (A.B2^T) ), both products in fp32
//          ref_kernel of problems/nvidia/nvfp4_dual_gemm/reference.py:27-77
//
// Structure (one CTA per SM, persistent, 7 warps):
//   warp 0      TMA producer: A/B tiles with 128-byte swizzle through
//               cp.async.bulk.tensor, the 128x4-blocked scale factors through
//               plain cp.async.bulk (each 128-row block of scales for a
//               256-wide K tile is one contiguous 2 KB run), into a ring of
//               kStages shared-memory stages guarded by full/empty mbarriers.
//   warp 6      scale copier: per K tile, tcgen05.cp moves the stage's scale
//               blocks into TMEM (32x128b, replicated to the four lane
//               quarters) and commits to sf_ready[stage].  Copies issued by
//               the MMA thread itself would serialise with its MMAs in the
//               tensor pipe (measured ~45 cycles per copy); from a second
//               thread they overlap with the MMAs.
//   warp 1      TMEM owner and MMA issuer: per K tile, four tcgen05.mma
//               kind::mxf4nvf4 (M=128, N=BN, K=64 each; two per step for the
//               dual GEMM, sharing the A tile) accumulate in fp32 in TMEM;
//               tcgen05.commit releases the stage and, after the last K tile,
//               hands the accumulator to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld rows of the accumulator(s), optional
//               silu(x)*y in fp32, fp16 conversion, 16-byte global stores.
// With BN=128 the GEMM double-buffers its accumulator in TMEM so the epilogue
// of tile i overlaps the main loop of tile i+1; BN=256 and the dual GEMM need
// all accumulator columns for one tile.  No load uses cluster multicast.
#include "common.cuh"
#include "kernels.h"

#include <cstdlib>

namespace nvfp4 {

constexpr int kBM = 128;
constexpr int kBK = 256;          // K elements per stage (128 bytes per row)
constexpr int kBKBytes = kBK / 2;
constexpr int kMmaK = 64;         // K per tcgen05.mma for kind::mxf4nvf4
constexpr int kSfBlockBytes = 512;  // one 128-row x 4-scale block
constexpr int kSfStageBytes = kSfBlockBytes * (kBK / kMmaK);  // 2 KB per operand per stage
constexpr int kThreads = 224;

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
  static constexpr int kTxBytes = kStageBytes + kSfOps * kSfStageBytes;
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
  int* status;
};

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

template <int BN, bool kDual>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_b2, const GemmParams p) {
  using Cfg = GemmConfig<BN, kDual>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;                                   // S x kStageBytes (1024-aligned each)
  uint8_t* sfbuf = smem + S * Cfg::kStageBytes;            // S x kSfOps x 2 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sfbuf + S * Cfg::kSfOps * kSfStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* sf_ready = bars + 2 * S;
  uint64_t* acc_full = bars + 3 * S;
  uint64_t* acc_empty = acc_full + Cfg::kAccBufs;
  uint64_t* drain = acc_empty + Cfg::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = p.K / kBK;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&sf_ready[s], 1);
    }
    for (int b = 0; b < Cfg::kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    mbar_init(drain + 1, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !abort_flag; t += gridDim.x) {
        int mb, nb, l;
        tile_coords(p, t, mb, nb, l);
        const uint8_t* sfa_src = p.sfa + l * p.sfa_lstride + static_cast<int64_t>(mb) * p.K * 8;
        const uint8_t* sfb_src = p.sfb + l * p.sfb_lstride + static_cast<int64_t>(nb) * (BN / 128) * p.K * 8;
        const uint8_t* sfb2_src =
            kDual ? p.sfb2 + l * p.sfb2_lstride + static_cast<int64_t>(nb) * (BN / 128) * p.K * 8 : nullptr;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            set_status(p.status, kStatusTimeoutEmpty);
            abort_flag = 1;
            break;
          }
          uint8_t* st = tiles + stage * Cfg::kStageBytes;
          uint8_t* sf = sfbuf + stage * Cfg::kSfOps * kSfStageBytes;
          mbar_arrive_expect_tx(&full[stage], Cfg::kTxBytes);
          tma_load_3d(st, &tm_a, &full[stage], kt * kBKBytes, mb * kBM, l, pol_a);
          tma_load_3d(st + Cfg::kABytes, &tm_b, &full[stage], kt * kBKBytes, nb * BN, l, pol_b);
          if (kDual) tma_load_3d(st + Cfg::kABytes + Cfg::kBBytes, &tm_b2, &full[stage], kt * kBKBytes, nb * BN, l, pol_b);
          bulk_load(sf, sfa_src + kt * kSfStageBytes, kSfStageBytes, &full[stage], pol_a);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            bulk_load(sf + (1 + j) * kSfStageBytes, sfb_src + static_cast<int64_t>(j) * p.K * 8 + kt * kSfStageBytes,
                      kSfStageBytes, &full[stage], pol_b);
          if (kDual) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              bulk_load(sf + (1 + BN / 128 + j) * kSfStageBytes,
                        sfb2_src + static_cast<int64_t>(j) * p.K * 8 + kt * kSfStageBytes, kSfStageBytes, &full[stage],
                        pol_b);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_nvf4(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !abort_flag; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1)) {
          set_status(p.status, kStatusTimeoutAccEmpty);
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * Cfg::kAccCols;
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&full[stage], phase) || !mbar_wait(&sf_ready[stage], phase)) {
            set_status(p.status, kStatusTimeoutFull);
            abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(tiles + stage * Cfg::kStageBytes);
          const uint32_t sfc = tmem_base + sf_col0 + stage * Cfg::kSfCols;
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk) {
            const uint64_t adesc = desc_kmajor_sw128(st + kk * (kMmaK / 2));
            const uint64_t bdesc = desc_kmajor_sw128(st + Cfg::kABytes + kk * (kMmaK / 2));
            const uint32_t accum = (kt | kk) != 0;
            mma_nvf4(d0, adesc, bdesc, idesc, sfc + 4 * kk, sfc + 16 + 4 * kk * (BN / 128), accum);
            if (kDual) {
              const uint64_t b2desc = desc_kmajor_sw128(st + Cfg::kABytes + Cfg::kBBytes + kk * (kMmaK / 2));
              mma_nvf4(d0 + BN, adesc, b2desc, idesc, sfc + 4 * kk, sfc + 16 + 16 * (BN / 128) + 4 * kk * (BN / 128),
                       accum);
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
        if (++acc == Cfg::kAccBufs) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Make sure every issued tcgen05 op has retired before TMEM is freed.
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------ scale copier
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const int total = ((p.num_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x)) * KT;
      for (int i = 0; i < total && !abort_flag; ++i) {
        if (!mbar_wait(&full[stage], phase)) {
          set_status(p.status, kStatusTimeoutFull);
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sf = smem_u32(sfbuf + stage * Cfg::kSfOps * kSfStageBytes);
        const uint32_t sfc = tmem_base + sf_col0 + stage * Cfg::kSfCols;
        // Per stage: SFA at columns [0,16) (MMA step kk at 4*kk), then per B
        // operand 16*(BN/128) columns where the scales of 128-row block j for
        // step kk sit at 4*(kk*(BN/128) + j), the column order an N=BN MMA
        // reads them in.
#pragma unroll
        for (int kk = 0; kk < kBK / kMmaK; ++kk)
          tmem_cp_32x128b_x4(sfc + 4 * kk, desc_sf_block(sf + kk * kSfBlockBytes));
#pragma unroll
        for (int op = 0; op < Cfg::kNB; ++op)
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
#pragma unroll
            for (int kk = 0; kk < kBK / kMmaK; ++kk)
              tmem_cp_32x128b_x4(sfc + 16 + op * 16 * (BN / 128) + 4 * (kk * (BN / 128) + j),
                                 desc_sf_block(sf + (1 + op * (BN / 128) + j) * kSfStageBytes + kk * kSfBlockBytes));
        tc_commit(&sf_ready[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      tc_commit(drain + 1);
      mbar_wait(drain + 1, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mb, nb, l;
      tile_coords(p, t, mb, nb, l);
      // All lanes must agree before the warp-collective tcgen05.ld below.
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase))) {
        if (lane == 0) set_status(p.status, kStatusTimeoutAccFull);
        abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mb * kBM + q * 32 + lane;
      __half* crow = p.c + l * p.c_lstride + static_cast<int64_t>(row) * p.ldc + static_cast<int64_t>(nb) * BN;
      const uint32_t tacc = tmem_base + acc * Cfg::kAccCols + (static_cast<uint32_t>(q * 32) << 16);
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
        }
        uint4 out[4];
        uint32_t* o = reinterpret_cast<uint32_t*>(out);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          __half2 h = __floats2half2_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          o[i] = *reinterpret_cast<uint32_t*>(&h);
        }
        uint4* dst = reinterpret_cast<uint4*>(crow + c0);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = out[i];
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == Cfg::kAccBufs) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
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
bool make_tma_3d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t L,
                    uint64_t row_stride, uint64_t lstride, uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {inner, rows, L};
  cuuint64_t strides[2] = {row_stride, lstride};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
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
  CUtensorMap ta, tb, tb2;
  const int K2 = g.K / 2;
  if (!make_operand_map(&ta, g.a, K2, g.M, g.L, g.a_lstride, kBM) ||
      !make_operand_map(&tb, g.b, K2, g.N, g.L, g.b_lstride, BN) ||
      (kDual && !make_operand_map(&tb2, g.b2, K2, g.N, g.L, g.b2_lstride, BN))) {
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
  const int grid = p.num_tiles < num_sms ? p.num_tiles : num_sms;
  gemm_kernel<BN, kDual><<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tb2, p);
  return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  static int forced_bn = -1;
  if (forced_bn < 0) {
    const char* e = getenv("NVFP4_GEMM_BN");
    forced_bn = e ? atoi(e) : 0;
  }
  const bool wide = forced_bn ? forced_bn == 256 && g.N % 256 == 0 : g.N % 256 == 0;
  if (wide) return launch_impl<256, false>(g, num_sms, stream, why);
  return launch_impl<128, false>(g, num_sms, stream, why);
}

cudaError_t launch_dual_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why) {
  return launch_impl<128, true>(g, num_sms, stream, why);
}

}  // namespace nvfp4
