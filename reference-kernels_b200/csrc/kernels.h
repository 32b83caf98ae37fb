// Host-side launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4 {

struct GemvParams {
  const uint8_t* a;    // [L][M][K/2] packed e2m1
  const uint8_t* b;    // [L][rows][K/2], row 0 used
  const uint8_t* sfa;  // [L][M][K/16] e4m3 codes, plain layout
  const uint8_t* sfb;  // [L][rows][K/16], row 0 used
  __half* c;           // [L][M]
  int M, K, L;
  int64_t a_lstride, b_lstride, sfa_lstride, sfb_lstride, c_lstride;  // elements of each array
  int ctas_per_l;                                                      // set by the launcher
};
cudaError_t launch_gemv(const GemvParams& in, int num_sms, cudaStream_t stream);

struct GemmArgs {
  const void *a, *b, *b2, *sfa, *sfb, *sfb2;
  void* c;
  int M, N, K, L;
  int64_t a_lstride, b_lstride, b2_lstride;        // bytes
  int64_t sfa_lstride, sfb_lstride, sfb2_lstride;  // bytes
  int64_t ldc, c_lstride;                          // elements
  int* status;                                     // device status word (bounded-wait timeouts)
};
cudaError_t launch_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why);
cudaError_t launch_dual_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why);

}  // namespace nvfp4
