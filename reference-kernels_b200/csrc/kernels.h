// Host-side launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include <cstdlib>

namespace nvfp4 {

// Launch with programmatic stream serialisation (the kernel calls pdl_wait()
// before touching global memory); optional cluster size.  NVFP4_PDL=0
// disables the attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       int cluster_x, Args&&... args) {
  static const bool pdl = [] {
    const char* e = getenv("NVFP4_PDL");
    return !(e && e[0] == '0');
  }();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

struct GemvParams {
  const uint8_t* a;    // [L][M][K/2] packed e2m1
  const uint8_t* b;    // [L][rows][K/2], row 0 used
  const uint8_t* sfa;  // blocked (128x4) e4m3 scales of A, batch l at + l * sfa_lstride
  const uint8_t* sfb;  // blocked scales of b (row block 0 used)
  __half* c;           // [L][M]
  int M, K, L;
  int64_t a_lstride, b_lstride, sfa_lstride, sfb_lstride, c_lstride;  // elements of each array
  int ctas_per_l;                                                      // set by the launcher
};
cudaError_t launch_gemv(const GemvParams& in, int num_sms, cudaStream_t stream);

// GEMV through TMA + tcgen05 (gemv_tc.cu); blocked scales; M % 128 == 0, K % 256 == 0.
struct GemvTcArgs {
  const void *a, *b, *sfa, *sfb;
  void* c;
  int M, K, L;
  int64_t a_lstride, b_lstride, sfa_lstride, sfb_lstride;  // bytes
  int64_t c_lstride;                                        // elements
  void* workspace;                                          // zero-initialised counters + partial sums
  size_t workspace_bytes;
  int* status;
  int inject;  // test hook: CTA 0 withholds its first A load (its pipeline waits then run out)
};
// Row blocks (M/128 * L) the tensor-core GEMV can track; larger calls use the SIMT GEMV.
constexpr int kGemvTcMaxCounterBlocks = 16384;
// Bytes of workspace the tensor-core GEMV needs (0 if the call is too large for it).
size_t gemv_tc_workspace_bytes(int M, int K, int L, int num_sms);
cudaError_t launch_gemv_tc(const GemvTcArgs& g, int num_sms, cudaStream_t stream, const char** why);

// Tuning / test switches from the environment (NVFP4_GEMM_BN, NVFP4_SPLITS,
// NVFP4_PAIR, NVFP4_STREAMK, NVFP4_PREFETCH, NVFP4_FAULT_INJECT,
// NVFP4_GEMV_PATH, NVFP4_GEMV_CTAS), read in one pass over `environ` per API call (six getenv
// calls cost ~1.5 us with a hundred-odd variables set).
struct EnvOptions {
  int gemm_bn = 0;       // 128 forces 128-wide tiles
  int splits = 0;        // > 0 forces the 1-CTA kernel's K splits
  int pair = -1;         // -1 default, 0 never 2-CTA tiles, 1 wherever the shape allows
  int streamk = 0;       // 0 default (off), -1 off, 1 hybrid, 2 pure
  int prefetch = 0;      // K tiles of B prefetched into L2
  int fault_inject = 0;  // test hook: CTA 0 withholds its first A load
  int gemv_simt = 0;     // NVFP4_GEMV_PATH=simt
  int gemv_ctas = 0;     // > 0 caps the tensor-core GEMV's CTA count (NVFP4_GEMV_CTAS)
  int b_evict = -1;      // L2 policy of B loads: -1 default, 0 evict_first, 1 normal, 2 evict_last
};
EnvOptions read_env_options();

struct GemmArgs {
  const void *a, *b, *b2, *sfa, *sfb, *sfb2;
  void* c;
  int M, N, K, L;
  int64_t a_lstride, b_lstride, b2_lstride;        // bytes
  int64_t sfa_lstride, sfb_lstride, sfb2_lstride;  // bytes
  int64_t ldc, c_lstride;                          // elements
  int* status;                                     // device status word (bounded-wait timeouts)
  int bn, splits, streamk, streamk_pure, pair;     // from gemm_plan
  int prefetch, inject;                            // from EnvOptions
  int b_evict;                                     // L2 policy of B loads (0 first, 1 normal, 2 last)
  void* workspace;                                 // stream-K partials + flags (zeroed once; left zeroed)
  size_t workspace_bytes;
};
struct GemmPlan {
  int bn;      // N tile: 128 or 256
  int splits;  // K splits per tile
  int streamk;  // 1: stream-K ranges over (tile, K tile) units (plain GEMM, tiles > SMs)
  int streamk_pure;  // 1: no whole-tile waves before the stream-K ranges (tests / comparison)
  int pair;     // 1: 2-CTA kernel, 256x256 tiles (plain GEMM, M % 256 == 0, N % 256 == 0, no split)
  size_t workspace_bytes;  // stream-K partial slots + flags; 0 otherwise (split K reduces on chip)
  int b_evict;             // L2 policy of B loads (0 evict_first, 1 normal, 2 evict_last)
};
GemmPlan gemm_plan(int M, int N, int K, int L, bool dual, int num_sms, const EnvOptions& opt);
cudaError_t launch_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why);
cudaError_t launch_dual_gemm(const GemmArgs& g, int num_sms, cudaStream_t stream, const char** why);

// Quantiser and scale-layout converter (quant.cu).
struct QuantArgs {
  const void* x;  // fp16 (dtype 0) or bf16 (dtype 1), [L][rows][K]
  int dtype;
  void* packed;  // [L][rows][K/2]
  void* sf_blk;  // blocked scales
  int rows, K, L;
  int64_t x_lstride;       // elements
  int64_t packed_lstride;  // bytes
  int64_t sf_lstride;      // bytes
  float global_scale;
};
cudaError_t launch_quantize(const QuantArgs& a, int num_sms, cudaStream_t stream);

struct ScaleLayoutArgs {
  const void* src;
  void* dst;
  int rows, sk, L;
  int64_t plain_row_stride, plain_lstride, blk_lstride;  // bytes
};
cudaError_t launch_scale_layout(const ScaleLayoutArgs& a, bool to_blocked, int num_sms, cudaStream_t stream);

}  // namespace nvfp4
