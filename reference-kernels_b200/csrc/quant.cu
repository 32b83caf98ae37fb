// NVFP4 producer kernels: quantisation of fp16 / bf16 data into the
// reference's input format, and conversion of block scales between the plain
// [rows][K/16] layout and the 128x4-blocked layout.
//
// Quantisation (one 16-element block of a row per thread):
//   amax  = max |x| over the block
//   s     = e4m3_rn_satfinite( amax / (6 * g) )          (g: global fp32 scale)
//   q_i   = e2m1_rn_satfinite( x_i / (float(s) * g) )    (all zero if s == 0)
// so that q_i * s * g approximates x_i; the values are written as packed
// e2m1 pairs (element 2j in the low nibble) and e4m3 scales already in the
// blocked layout that tcgen05.mma and the reference's "permuted" tensors use.
// This is the producer step that generate_input performs with an
// advanced-index scatter (problems/nvidia/nvfp4_gemm/reference.py:103-152);
// the blocked order is to_blocked (reference.py:12-24).  Both are
// element-wise, HBM-bound kernels (32 B read + 9 B written per block).
#include <cuda_bf16.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {

__device__ __forceinline__ int64_t blk_off(int i, int j, int sk) {
  return static_cast<int64_t>(i >> 7) * (sk >> 2) * 512 + (j >> 2) * 512 + (i & 31) * 16 + ((i & 127) >> 5) * 4 + (j & 3);
}

// e2m1 pair: `lo` goes to the low nibble.
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint16_t q;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u16.u8 %0, t;\n\t}" : "=h"(q) : "f"(hi), "f"(lo));
  return q;
}

__device__ __forceinline__ uint32_t e4m3_byte(float v) {
  uint16_t s;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(s) : "f"(0.f), "f"(v));
  return s & 0xFF;
}

__device__ __forceinline__ float e4m3_value(uint32_t code) {
  const uint32_t h = e4m3x2_to_f16x2(static_cast<uint16_t>(code));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFF)));
}

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&v)[16]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  const uint4 a = q[0], b = q[1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<T, __half>::value) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    } else {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ x, uint8_t* __restrict__ q,
                                                       uint8_t* __restrict__ sf, int rows, int K, int L,
                                                       int64_t x_lstride, int64_t q_lstride, int64_t sf_lstride,
                                                       float gscale) {
  if (threadIdx.x == 0) pdl_allow_dependents();
  pdl_wait();
  const int sk = K >> 4;
  const int64_t per_l = static_cast<int64_t>(rows) * sk;
  const int64_t total = per_l * L;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int l = static_cast<int>(t / per_l);
    const int64_t r = t - l * per_l;
    const int i = static_cast<int>(r / sk), j = static_cast<int>(r - static_cast<int64_t>(i) * sk);
    float v[16];
    load16(x + l * x_lstride + static_cast<int64_t>(i) * K + j * 16, v);
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
    const uint32_t code = e4m3_byte(__fdiv_rn(amax, 6.f * gscale));
    const float d = e4m3_value(code) * gscale;
    uint32_t packed[2] = {0u, 0u};
    if (d > 0.f) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        packed[e >> 2] |= e2m1x2(__fdiv_rn(v[2 * e], d), __fdiv_rn(v[2 * e + 1], d)) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2*>(q + l * q_lstride + static_cast<int64_t>(i) * (K >> 1) + j * 8) =
        make_uint2(packed[0], packed[1]);
    sf[l * sf_lstride + blk_off(i, j, sk)] = static_cast<uint8_t>(code);
  }
}

// One thread per 4 consecutive scales of a row (one aligned 32-bit word in
// both layouts).
template <bool kToBlocked>
__global__ void __launch_bounds__(256) scale_layout_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                           int rows, int sk, int L, int64_t plain_row_stride,
                                                           int64_t plain_lstride, int64_t blk_lstride) {
  if (threadIdx.x == 0) pdl_allow_dependents();
  pdl_wait();
  const int words = sk >> 2;
  const int64_t per_l = static_cast<int64_t>(rows) * words;
  const int64_t total = per_l * L;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int l = static_cast<int>(t / per_l);
    const int64_t r = t - l * per_l;
    const int i = static_cast<int>(r / words), w = static_cast<int>(r - static_cast<int64_t>(i) * words);
    const int64_t p = l * plain_lstride + i * plain_row_stride + 4 * w;
    const int64_t b = l * blk_lstride + blk_off(i, 4 * w, sk);
    if (kToBlocked)
      *reinterpret_cast<uint32_t*>(dst + b) = *reinterpret_cast<const uint32_t*>(src + p);
    else
      *reinterpret_cast<uint32_t*>(dst + p) = *reinterpret_cast<const uint32_t*>(src + b);
  }
}

static int grid_for(int64_t items, int num_sms) {
  int64_t g = (items + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  return static_cast<int>(g < cap ? (g < 1 ? 1 : g) : cap);
}

cudaError_t launch_quantize(const QuantArgs& a, int num_sms, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(a.rows) * (a.K / 16) * a.L;
  const dim3 grid(grid_for(items, num_sms)), block(256);
  if (a.dtype == 0)
    return launch_pdl(quantize_kernel<__half>, grid, block, 0, stream, 1, static_cast<const __half*>(a.x),
                      static_cast<uint8_t*>(a.packed), static_cast<uint8_t*>(a.sf_blk), a.rows, a.K, a.L,
                      a.x_lstride, a.packed_lstride, a.sf_lstride, a.global_scale);
  return launch_pdl(quantize_kernel<__nv_bfloat16>, grid, block, 0, stream, 1,
                    static_cast<const __nv_bfloat16*>(a.x), static_cast<uint8_t*>(a.packed),
                    static_cast<uint8_t*>(a.sf_blk), a.rows, a.K, a.L, a.x_lstride, a.packed_lstride, a.sf_lstride,
                    a.global_scale);
}

cudaError_t launch_scale_layout(const ScaleLayoutArgs& a, bool to_blocked, int num_sms, cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(a.rows) * (a.sk / 4) * a.L;
  const dim3 grid(grid_for(items, num_sms)), block(256);
  if (to_blocked)
    return launch_pdl(scale_layout_kernel<true>, grid, block, 0, stream, 1, static_cast<const uint8_t*>(a.src),
                      static_cast<uint8_t*>(a.dst), a.rows, a.sk, a.L, a.plain_row_stride, a.plain_lstride,
                      a.blk_lstride);
  return launch_pdl(scale_layout_kernel<false>, grid, block, 0, stream, 1, static_cast<const uint8_t*>(a.src),
                    static_cast<uint8_t*>(a.dst), a.rows, a.sk, a.L, a.plain_row_stride, a.plain_lstride,
                    a.blk_lstride);
}

}  // namespace nvfp4
