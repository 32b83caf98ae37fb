// nvfp4_gemv_noalloc: the tensor-core GEMV with its scratch memory in a
// fixed, library-owned device array instead of a workspace obtained with
// cudaMalloc.
//
// Some callers cannot allocate device memory at call time: code running
// under an allocator that forbids it (a memory pool that is already fully
// reserved, a process that must never grow its footprint after start-up),
// or host code that has no access to cudaMalloc at all.  For them this entry
// point uses only the static array below.  The array is part of the library
// image: every GPU that loads the library holds kNoAllocScratchBytes of it
// until the process exits.
#include <mutex>

#include "../../include/nvfp4_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace nvfp4 {

// 4 MiB: the arrival counters (kGemvTcMaxCounterBlocks ints) plus partial sums
// for about 7,800 (row block x contributor) pairs -- enough for every shape of
// the reference's GEMV tests and benchmarks and for BASELINE's M=7168 K=16384 L=4.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

static __device__ __align__(256) uint8_t g_gemv_scratch[kNoAllocScratchBytes];

namespace {

// Device address of g_gemv_scratch on each device.  In host code the symbol
// name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, taken once per device with that device current.
void* g_scratch_addr[64] = {nullptr};
int g_num_sms[64] = {0};
std::mutex g_setup_mutex;

// First call on a device: look up the array's device address and the SM
// count, and zero the arrival counters once (synchronously, which is why the
// first call must not be inside a stream capture).  Later calls rely on the
// kernel leaving every counter it used back at zero.
cudaError_t setup_device(int dev) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev]) return cudaSuccess;
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_gemv_scratch);
  if (e != cudaSuccess) return e;
  int n = 0;
  e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  e = cudaMemset(ptr, 0, sizeof(int) * kGemvTcMaxCounterBlocks);
  if (e != cudaSuccess) return e;
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  g_num_sms[dev] = n > 0 ? n : 148;
  g_scratch_addr[dev] = ptr;
  return cudaSuccess;
}

}  // namespace

int* device_status_word(int dev);  // capi.cu

// Called by nvfp4_device_status(clear) after a recorded timeout: a GEMV that
// gave up may have left its arrival counters non-zero.
void noalloc_scratch_reset(int dev) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (dev >= 0 && dev < 64 && g_scratch_addr[dev])
    cudaMemset(g_scratch_addr[dev], 0, sizeof(int) * kGemvTcMaxCounterBlocks);
}
}  // namespace nvfp4

using namespace nvfp4;

// Records the message that nvfp4_last_error() returns (defined in capi.cu).
int nvfp4_record_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
#define noalloc_fail nvfp4_record_error

static_assert(kNoAllocScratchBytes == NVFP4_GEMV_NOALLOC_SCRATCH_BYTES, "header constant");

extern "C" __attribute__((visibility("default"))) int nvfp4_gemv_noalloc(
    const void* a, const void* b, const void* sfa_blk, const void* sfb_blk, void* c, int M, int K, int L,
    int64_t a_lstride, int64_t b_lstride, int64_t sfa_lstride, int64_t sfb_lstride, int64_t c_lstride,
    void* stream) {
  if (!a || !b || !sfa_blk || !sfb_blk || !c) return noalloc_fail(NVFP4_ERR_NULL, "nvfp4_gemv_noalloc: null pointer");
  if (M <= 0 || K <= 0 || L <= 0 || M % 128 != 0 || K % 256 != 0)
    return noalloc_fail(NVFP4_ERR_SHAPE,
                        "nvfp4_gemv_noalloc: needs M %% 128 == 0 and K %% 256 == 0 (got M=%d K=%d L=%d)", M, K, L);
  const uintptr_t mis = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                        reinterpret_cast<uintptr_t>(sfa_blk) | reinterpret_cast<uintptr_t>(sfb_blk);
  if ((mis & 15) || (reinterpret_cast<uintptr_t>(c) & 1) || (a_lstride % 16) || (b_lstride % 16) ||
      (sfa_lstride % 16) || (sfb_lstride % 16))
    return noalloc_fail(NVFP4_ERR_ALIGN,
                        "nvfp4_gemv_noalloc: operands and scales need 16-byte aligned bases and batch strides");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return noalloc_fail(NVFP4_ERR_DEVICE, "nvfp4_gemv_noalloc: no usable CUDA device");
  cudaError_t e = setup_device(dev);
  if (e != cudaSuccess)
    return noalloc_fail(NVFP4_ERR_CUDA, "nvfp4_gemv_noalloc: cudaGetSymbolAddress of the scratch array failed: %s",
                        cudaGetErrorString(e));
  const size_t need = gemv_tc_workspace_bytes(M, K, L, g_num_sms[dev]);
  if (need == 0)
    return noalloc_fail(NVFP4_ERR_SHAPE,
                        "nvfp4_gemv_noalloc: M=%d L=%d gives %lld 128-row blocks, more than the %d arrival "
                        "counters of the fixed scratch array",
                        M, L, static_cast<long long>(M / 128) * L, kGemvTcMaxCounterBlocks);
  if (need > kNoAllocScratchBytes)
    return noalloc_fail(NVFP4_ERR_SHAPE,
                        "nvfp4_gemv_noalloc: M=%d K=%d L=%d needs %zu bytes of scratch, more than the fixed %zu",
                        M, K, L, need, kNoAllocScratchBytes);
  int* status = device_status_word(dev);
  if (!status)
    return noalloc_fail(NVFP4_ERR_CUDA, "nvfp4_gemv_noalloc: cannot look up the device status word");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GemvTcArgs g{};
  g.a = a;
  g.b = b;
  g.sfa = sfa_blk;
  g.sfb = sfb_blk;
  g.c = c;
  g.M = M;
  g.K = K;
  g.L = L;
  g.a_lstride = a_lstride;
  g.b_lstride = b_lstride;
  g.sfa_lstride = sfa_lstride;
  g.sfb_lstride = sfb_lstride;
  g.c_lstride = c_lstride;
  g.workspace = g_scratch_addr[dev];
  g.workspace_bytes = kNoAllocScratchBytes;
  g.status = status;
  const char* why = nullptr;
  e = launch_gemv_tc(g, g_num_sms[dev], s, &why);
  if (e != cudaSuccess)
    return noalloc_fail(NVFP4_ERR_CUDA, "nvfp4_gemv_noalloc: %s", why ? why : cudaGetErrorString(e));
  return NVFP4_OK;
}
