// NVFP4 block-scaled GEMV for sm_100a:  c[m, l] = sum_k (a[m,k,l] sfa[m,k/16,l]) (b[k,l] sfb[k/16,l])
//
// Semantics follow ref_kernel of problems/nvidia/nvfp4_gemv/reference.py:28-54
// (column 0 of a block-scaled GEMM with fp32 accumulation, fp16 output).
//
// The kernel is HBM-bound on the packed A stream (K/2 bytes per row plus K/16
// scale bytes), so it is written as a streaming kernel, not a tensor-core one:
//   * one persistent CTA range of rows per (CTA, l); ranges differ by at most
//     one quad of rows, so every SM streams the same number of bytes;
//   * within a CTA the warps split K into 512-byte segments (one 16-byte
//     ld.global.nc per lane per row) and every warp streams up to 8 rows at
//     once, so each lane keeps eight 128-bit loads in flight;
//   * scales are read from the 128x4-blocked layout (the same tensors the
//     tensor-core path reads);
//   * e2m1 pairs are widened with cvt.rn.f16x2.e2m1x2 and multiplied against
//     the (unscaled) e2m1 values of b with HFMA2: the products of two e2m1
//     values are multiples of 1/4 below 36, so the 8-term sums per f16 half
//     are exact; the group sum is then scaled in fp32 by sfa*sfb (an exact
//     product of two e4m3 values) and accumulated in fp32;
//   * per-warp partial sums are folded across lanes with a 9-shuffle
//     halving butterfly and across warps through shared memory.
#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {



constexpr int kGemvRowsPerBatch = 8;
constexpr int kGemvMaxWarps = 16;

__device__ __forceinline__ uint4 ld_stream_16(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Dot product of 32 e2m1 values (16 bytes) with 32 f16 values of b for two
// 16-element groups; returns group sums g0, g1 (exact, in fp32).
__device__ __forceinline__ float2 group_sums(const uint4 av, const uint32_t (&bh)[16]) {
  const uint32_t w[4] = {av.x, av.y, av.z, av.w};
  __half2 acc0 = __float2half2_rn(0.f), acc1 = __float2half2_rn(0.f);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint32_t h[4];
    e2m1x8_to_f16x2x4(w[i], h);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      acc0 = __hfma2(*reinterpret_cast<__half2*>(&h[j]), *reinterpret_cast<const __half2*>(&bh[i * 4 + j]), acc0);
  }
#pragma unroll
  for (int i = 2; i < 4; ++i) {
    uint32_t h[4];
    e2m1x8_to_f16x2x4(w[i], h);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      acc1 = __hfma2(*reinterpret_cast<__half2*>(&h[j]), *reinterpret_cast<const __half2*>(&bh[i * 4 + j]), acc1);
  }
  const float2 f0 = __half22float2(acc0), f1 = __half22float2(acc1);
  return make_float2(f0.x + f0.y, f1.x + f1.y);
}

__device__ __forceinline__ float2 e4m3_pair(uint16_t codes) {
  uint32_t h = e4m3x2_to_f16x2(codes);
  return __half22float2(*reinterpret_cast<__half2*>(&h));
}

// Byte offset of scale (row i, group j) in the 128x4-blocked layout
// (to_blocked of problems/nvidia/nvfp4_gemv/reference.py:14-25).  Groups 2t
// and 2t+1 share one aligned 16-bit word.
__device__ __forceinline__ int64_t blocked_offset(int i, int j, int sk) {
  return static_cast<int64_t>(i >> 7) * (sk >> 2) * 512 + (j >> 2) * 512 + (i & 31) * 16 + ((i & 127) >> 5) * 4 + (j & 3);
}

// One work item = (batch of up to 8 rows, one 512-byte K segment of this warp).
struct GemvItem {
  uint4 av[kGemvRowsPerBatch];
  uint16_t sa[kGemvRowsPerBatch];
};

__device__ __forceinline__ void load_item(GemvItem& it, const uint8_t* a_l, const uint8_t* sfa_l, int row0, int nrows,
                                          int kb, int K2, int SK) {
#pragma unroll
  for (int r = 0; r < kGemvRowsPerBatch; ++r) {
    if (r < nrows && kb < K2) {
      it.av[r] = ld_stream_16(a_l + static_cast<int64_t>(row0 + r) * K2 + kb);
      it.sa[r] = __ldg(reinterpret_cast<const uint16_t*>(sfa_l + blocked_offset(row0 + r, kb >> 3, SK)));
    } else {
      it.av[r] = make_uint4(0, 0, 0, 0);
      it.sa[r] = 0;
    }
  }
}

__global__ void __launch_bounds__(kGemvMaxWarps * 32) gemv_kernel(const GemvParams p) {
  __shared__ float red[2][kGemvMaxWarps][kGemvRowsPerBatch];
  if (threadIdx.x == 0) pdl_allow_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int l = blockIdx.y;
  const int K2 = p.K >> 1, SK = p.K >> 4;
  const int nseg = (K2 + 511) >> 9;
  const int my_segs = (nseg - warp + nwarps - 1) / nwarps;  // segments seg = warp + j*nwarps

  // Row range of this CTA, in quads of rows.
  const int quads = p.M >> 2;
  const int q0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * quads) / p.ctas_per_l);
  const int q1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * quads) / p.ctas_per_l);
  const int nbatch = (q1 - q0 + 1) >> 1;

  const uint8_t* a_l = p.a + l * p.a_lstride;
  const uint8_t* sfa_l = p.sfa + l * p.sfa_lstride;
  const uint8_t* b_l = p.b + l * p.b_lstride;
  const uint8_t* sfb_l = p.sfb + l * p.sfb_lstride;

  // b of the current segment (unscaled e2m1 as f16 pairs) and its two scales.
  uint32_t bh[16];
  float sb0 = 0.f, sb1 = 0.f;
  int cached_seg = -1;

  // Items are visited batch-major, segment-minor; item i+1 is loaded while
  // item i is being reduced, so every lane keeps 8 loads in flight across the
  // per-batch barrier.
  const int nitems = nbatch * my_segs;
  GemvItem cur, nxt;
  auto item_coords = [&](int i, int& row0, int& nrows, int& seg) {
    const int bi = i / my_segs;
    const int j = i - bi * my_segs;
    const int qb = q0 + 2 * bi;
    row0 = qb * 4;
    nrows = (q1 - qb >= 2) ? 8 : 4;
    seg = warp + j * nwarps;
  };
  if (nitems > 0) {
    int row0, nrows, seg;
    item_coords(0, row0, nrows, seg);
    load_item(cur, a_l, sfa_l, row0, nrows, seg * 512 + lane * 16, K2, SK);
  }
  float part[kGemvRowsPerBatch];
#pragma unroll
  for (int r = 0; r < kGemvRowsPerBatch; ++r) part[r] = 0.f;
  int buf = 0;
  // Warps with no segment (nseg < nwarps never happens; guard anyway) still join the barriers.
  const int total_batches = nbatch;
  int item = 0;
  for (int bi = 0; bi < total_batches; ++bi) {
    int row0 = (q0 + 2 * bi) * 4;
    const int nrows = (q1 - (q0 + 2 * bi) >= 2) ? 8 : 4;
    for (int j = 0; j < my_segs; ++j, ++item) {
      if (item + 1 < nitems) {
        int r1, n1, s1;
        item_coords(item + 1, r1, n1, s1);
        load_item(nxt, a_l, sfa_l, r1, n1, s1 * 512 + lane * 16, K2, SK);
      }
      const int seg = warp + j * nwarps;
      const int kb = seg * 512 + lane * 16;
      if (kb < K2) {
        if (seg != cached_seg) {
          const uint4 bv = *reinterpret_cast<const uint4*>(b_l + kb);
          const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t h[4];
            e2m1x8_to_f16x2x4(bw[i], h);
#pragma unroll
            for (int q = 0; q < 4; ++q) bh[i * 4 + q] = h[q];
          }
          const float2 sb = e4m3_pair(*reinterpret_cast<const uint16_t*>(sfb_l + blocked_offset(0, kb >> 3, SK)));
          sb0 = sb.x;
          sb1 = sb.y;
          cached_seg = seg;
        }
#pragma unroll
        for (int r = 0; r < kGemvRowsPerBatch; ++r) {
          const float2 g = group_sums(cur.av[r], bh);
          const float2 s = e4m3_pair(cur.sa[r]);
          part[r] = fmaf(g.x, s.x * sb0, part[r]);
          part[r] = fmaf(g.y, s.y * sb1, part[r]);
        }
      }
      cur = nxt;
    }

    // Halving butterfly: after it, lane j holds the warp total of row
    // 4*bit4(j) + 2*bit3(j) + bit2(j).
    const bool up16 = lane & 16, up8 = lane & 8, up4 = lane & 4;
    float v4[4], v2[2], v1;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = up16 ? part[i] : part[4 + i];
      const float keep = up16 ? part[4 + i] : part[i];
      v4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = up8 ? v4[i] : v4[2 + i];
      const float keep = up8 ? v4[2 + i] : v4[i];
      v2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    {
      const float send = up4 ? v2[0] : v2[1];
      const float keep = up4 ? v2[1] : v2[0];
      v1 = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
    v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
    if ((lane & 3) == 0) red[buf][warp][(up16 ? 4 : 0) + (up8 ? 2 : 0) + (up4 ? 1 : 0)] = v1;
#pragma unroll
    for (int r = 0; r < kGemvRowsPerBatch; ++r) part[r] = 0.f;
    __syncthreads();
    if (threadIdx.x < nrows) {
      float s = 0.f;
      for (int w = 0; w < nwarps; ++w) s += red[buf][w][threadIdx.x];
      p.c[l * p.c_lstride + row0 + threadIdx.x] = __float2half_rn(s);
    }
    buf ^= 1;
  }
}

// Host launcher (called from the C ABI in capi.cu).  The grid is exactly the
// number of CTAs that can be resident at once, split evenly over the L batch
// indices, so every CTA streams the same number of rows in a single wave.
cudaError_t launch_gemv(const GemvParams& in, int num_sms, cudaStream_t stream) {
  GemvParams p = in;
  const int K2 = p.K / 2;
  const int nseg = (K2 + 511) / 512;
  const int nwarps = nseg < kGemvMaxWarps ? nseg : kGemvMaxWarps;
  static int occ_cache[kGemvMaxWarps + 1] = {0};
  if (!occ_cache[nwarps]) {
    int occ = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_kernel, nwarps * 32, 0);
    if (e != cudaSuccess) return e;
    occ_cache[nwarps] = occ > 0 ? occ : 1;
  }
  int ctas_per_sm = occ_cache[nwarps];
  // More than ~48 warps per SM only adds barrier traffic.
  while (ctas_per_sm > 1 && ctas_per_sm * nwarps > 48) --ctas_per_sm;
  const int total = num_sms * ctas_per_sm;
  int per_l = total / p.L;
  if (per_l < 1) per_l = 1;
  const int quads = p.M / 4;
  if (per_l > quads) per_l = quads;
  p.ctas_per_l = per_l;
  dim3 grid(per_l, p.L), block(nwarps * 32);
  return launch_pdl(gemv_kernel, grid, block, 0, stream, 1, p);
}

}  // namespace nvfp4
