// C ABI of libnvfp4_b200.so: plain pointers, sizes and strides; no torch types.
// Declarations and the reference interface each entry point replaces are in
// include/nvfp4_b200.h.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "../../include/nvfp4_b200.h"

using namespace nvfp4;


static thread_local char g_err[512] = "";

static int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int nvfp4_record_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// One device-resident status word per device; kernels record bounded-wait
// timeouts here (0 = ok).
static __device__ int g_status_word;

namespace nvfp4 {
// Address of the status word on `dev` (the current device); nullptr if it
// cannot be looked up.  Shared with the allocation-free GEMV entry point.
int* device_status_word(int dev);
void noalloc_scratch_reset(int dev);
}  // namespace nvfp4

static int* status_ptr(int dev) { return nvfp4::device_status_word(dev); }

int* nvfp4::device_status_word(int dev) {
  static int* ptrs[64] = {nullptr};
  if (dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

static int num_sms_of(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// Per-device workspaces for kernels that combine partial results across CTAs
// (kind 0: the tensor-core GEMV; kind 1: the stream-K GEMM).  Allocated on the first call that needs it (and
// grown when a later call needs more), zeroed once; the kernels leave it
// zeroed.  Calls on one device share it, so they must not overlap on the GPU.
struct DeviceWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
enum { kWsGemv = 0, kWsGemm = 1 };
static DeviceWorkspace g_ws[2][64];
static std::mutex g_ws_mutex;

static void* workspace_for(int kind, int dev, size_t bytes, cudaStream_t stream, cudaError_t* err) {
  *err = cudaSuccess;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  DeviceWorkspace& w = g_ws[kind][dev];
  if (w.bytes >= bytes) return w.ptr;
  // Growing the workspace synchronises the device and allocates, neither of
  // which a stream capture allows: make one uncaptured call of the largest
  // shape first.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone) {
    *err = cudaErrorStreamCaptureUnsupported;
    return nullptr;
  }
  if (w.ptr) {
    // earlier launches may still read the old buffer
    if ((*err = cudaDeviceSynchronize()) != cudaSuccess) return nullptr;
    cudaFree(w.ptr);
    w.ptr = nullptr;
    w.bytes = 0;
  }
  size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
  if ((*err = cudaMalloc(&w.ptr, want)) != cudaSuccess) return nullptr;
  if ((*err = cudaMemsetAsync(w.ptr, 0, want, stream)) != cudaSuccess) return nullptr;
  w.bytes = want;
  return w.ptr;
}

extern "C" char** environ;

namespace nvfp4 {
EnvOptions read_env_options() {
  EnvOptions o;
  for (char** e = environ; e && *e; ++e) {
    const char* v = *e;
    if (strncmp(v, "NVFP4_", 6) != 0) continue;
    v += 6;
    auto key = [&](const char* k) -> const char* {  // value if v is "k=..."
      const size_t n = strlen(k);
      return (strncmp(v, k, n) == 0 && v[n] == '=') ? v + n + 1 : nullptr;
    };
    const char* x;
    if ((x = key("GEMM_BN"))) o.gemm_bn = atoi(x);
    else if ((x = key("SPLITS"))) o.splits = atoi(x);
    else if ((x = key("PAIR"))) o.pair = (x[0] == '0') ? 0 : (x[0] == '1') ? 1 : -1;
    else if ((x = key("STREAMK"))) o.streamk = atoi(x);
    else if ((x = key("PREFETCH"))) o.prefetch = atoi(x);
    else if ((x = key("FAULT_INJECT"))) o.fault_inject = (x[0] == '1');
    else if ((x = key("GEMV_PATH"))) o.gemv_simt = (strcmp(x, "simt") == 0);
    else if ((x = key("GEMV_CTAS"))) o.gemv_ctas = atoi(x);
    else if ((x = key("B_EVICT"))) o.b_evict = atoi(x);
  }
  return o;
}
}  // namespace nvfp4

static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

#define NVFP4_API extern "C" __attribute__((visibility("default")))

NVFP4_API const char* nvfp4_last_error(void) { return g_err; }

NVFP4_API int nvfp4_abi_version(void) { return 2; }

NVFP4_API int nvfp4_device_status(int clear) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_status_word, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    // A bounded wait ran out: the kernel that gave up may have left arrival
    // counters, stream-K flags or partial sums in the shared workspaces.  Wait
    // for the device, then zero every workspace of this device (and the
    // allocation-free GEMV's scratch) so that the next call starts clean.
    cudaDeviceSynchronize();
    {
      std::lock_guard<std::mutex> lock(g_ws_mutex);
      for (int kind = 0; kind < 2; ++kind)
        if (dev >= 0 && dev < 64 && g_ws[kind][dev].ptr) cudaMemset(g_ws[kind][dev].ptr, 0, g_ws[kind][dev].bytes);
    }
    nvfp4::noalloc_scratch_reset(dev);
    const int zero = 0;
    cudaMemcpyToSymbol(g_status_word, &zero, sizeof(int));
    cudaDeviceSynchronize();
  }
  return v;
}

NVFP4_API int nvfp4_gemv(const void* a, const void* b, const void* sfa_blk, const void* sfb_blk, void* c, int M,
                         int K, int L, int64_t a_lstride, int64_t b_lstride, int64_t sfa_lstride, int64_t sfb_lstride,
                         int64_t c_lstride, void* stream) {
  if (!a || !b || !sfa_blk || !sfb_blk || !c) return fail(NVFP4_ERR_NULL, "nvfp4_gemv: null pointer");
  if (M <= 0 || K <= 0 || L <= 0) return fail(NVFP4_ERR_SHAPE, "nvfp4_gemv: M, K, L must be positive");
  if (M % 128 != 0) return fail(NVFP4_ERR_SHAPE, "nvfp4_gemv: M=%d must be a multiple of 128", M);
  if (K % 64 != 0) return fail(NVFP4_ERR_SHAPE, "nvfp4_gemv: K=%d must be a multiple of 64", K);
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(sfa_blk, 16) || !aligned(sfb_blk, 16) || !aligned(c, 2) ||
      (a_lstride % 16) || (b_lstride % 16) || (sfa_lstride % 16) || (sfb_lstride % 16))
    return fail(NVFP4_ERR_ALIGN, "nvfp4_gemv: operands and scales need 16-byte aligned bases and batch strides");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4_ERR_DEVICE, "nvfp4_gemv: no CUDA device");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const EnvOptions opt = read_env_options();
  const int ctas = (opt.gemv_ctas > 0 && opt.gemv_ctas < num_sms_of(dev)) ? opt.gemv_ctas : num_sms_of(dev);
  const bool simt = (K % 256 != 0) || opt.gemv_simt || gemv_tc_workspace_bytes(M, K, L, ctas) == 0;
  if (!simt) {
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
    g.workspace_bytes = gemv_tc_workspace_bytes(M, K, L, ctas);
    cudaError_t e = cudaSuccess;
    g.workspace = workspace_for(kWsGemv, dev, g.workspace_bytes, s, &e);
    if (!g.workspace)
      return fail(NVFP4_ERR_CUDA, "nvfp4_gemv: workspace: %s",
                  e == cudaErrorStreamCaptureUnsupported
                      ? "it must grow, which a stream capture does not allow; make one uncaptured call of this shape "
                        "first"
                      : cudaGetErrorString(e));
    g.status = status_ptr(dev);
    g.inject = opt.fault_inject;
    const char* why = nullptr;
    e = launch_gemv_tc(g, ctas, s, &why);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "nvfp4_gemv: %s", why ? why : cudaGetErrorString(e));
    return NVFP4_OK;
  }
  GemvParams p;
  p.a = static_cast<const uint8_t*>(a);
  p.b = static_cast<const uint8_t*>(b);
  p.sfa = static_cast<const uint8_t*>(sfa_blk);
  p.sfb = static_cast<const uint8_t*>(sfb_blk);
  p.c = static_cast<__half*>(c);
  p.M = M;
  p.K = K;
  p.L = L;
  p.a_lstride = a_lstride;
  p.b_lstride = b_lstride;
  p.sfa_lstride = sfa_lstride;
  p.sfb_lstride = sfb_lstride;
  p.c_lstride = c_lstride;
  p.ctas_per_l = 1;
  cudaError_t e = launch_gemv(p, num_sms_of(dev), s);
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "nvfp4_gemv: launch failed: %s", cudaGetErrorString(e));
  return NVFP4_OK;
}

static int check_gemm_common(const char* name, const void* a, const void* b, const void* sfa, const void* sfb,
                             const void* c, int M, int N, int K, int L, int64_t a_lstride, int64_t b_lstride,
                             int64_t sfa_lstride, int64_t sfb_lstride, int64_t ldc, int64_t c_lstride) {
  if (!a || !b || !sfa || !sfb || !c) return fail(NVFP4_ERR_NULL, "%s: null pointer", name);
  if (M <= 0 || N <= 0 || K <= 0 || L <= 0) return fail(NVFP4_ERR_SHAPE, "%s: sizes must be positive", name);
  if (M % 128 || N % 128)
    return fail(NVFP4_ERR_SHAPE, "%s: M=%d and N=%d must be multiples of 128", name, M, N);
  if (K % 64) return fail(NVFP4_ERR_SHAPE, "%s: K=%d must be a multiple of 64", name, K);
  if (ldc < N) return fail(NVFP4_ERR_SHAPE, "%s: ldc=%lld < N=%d", name, (long long)ldc, N);
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(sfa, 16) || !aligned(sfb, 16) || !aligned(c, 16) ||
      (a_lstride % 16) || (b_lstride % 16) || (sfa_lstride % 16) || (sfb_lstride % 16) || (ldc % 8) ||
      (c_lstride % 8))
    return fail(NVFP4_ERR_ALIGN,
                "%s: operands and scales need 16-byte aligned bases and batch strides; ldc and the C batch "
                "stride must be multiples of 8",
                name);
  return NVFP4_OK;
}

// Copies a GEMM plan into the launch arguments and attaches the stream-K
// workspace when the plan needs one.
static int apply_plan(const char* who, int dev, const GemmPlan& pl, GemmArgs& g, void* stream) {
  g.bn = pl.bn;
  g.splits = pl.splits;
  g.streamk = pl.streamk;
  g.streamk_pure = pl.streamk_pure;
  g.pair = pl.pair;
  if (pl.workspace_bytes) {
    cudaError_t we;
    g.workspace = workspace_for(kWsGemm, dev, pl.workspace_bytes, static_cast<cudaStream_t>(stream), &we);
    if (!g.workspace)
      return fail(NVFP4_ERR_CUDA, "%s: workspace: %s", who,
                  we == cudaErrorStreamCaptureUnsupported
                      ? "it must grow, which a stream capture does not allow; make one uncaptured call of this shape "
                        "first"
                      : cudaGetErrorString(we));
    g.workspace_bytes = pl.workspace_bytes;
  }
  return NVFP4_OK;
}

NVFP4_API int nvfp4_gemm(const void* a, const void* b, const void* sfa_blk, const void* sfb_blk, void* c, int M, int N, int K,
               int L, int64_t a_lstride, int64_t b_lstride, int64_t sfa_lstride, int64_t sfb_lstride, int64_t ldc,
               int64_t c_lstride, void* stream) {
  int rc = check_gemm_common("nvfp4_gemm", a, b, sfa_blk, sfb_blk, c, M, N, K, L, a_lstride, b_lstride, sfa_lstride,
                             sfb_lstride, ldc, c_lstride);
  if (rc) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4_ERR_DEVICE, "nvfp4_gemm: no CUDA device");
  GemmArgs g{};
  g.a = a;
  g.b = b;
  g.b2 = b;
  g.sfa = sfa_blk;
  g.sfb = sfb_blk;
  g.sfb2 = sfb_blk;
  g.c = c;
  g.M = M;
  g.N = N;
  g.K = K;
  g.L = L;
  g.a_lstride = a_lstride;
  g.b_lstride = b_lstride;
  g.b2_lstride = b_lstride;
  g.sfa_lstride = sfa_lstride;
  g.sfb_lstride = sfb_lstride;
  g.sfb2_lstride = sfb_lstride;
  g.ldc = ldc;
  g.c_lstride = c_lstride;
  g.status = status_ptr(dev);
  const EnvOptions opt = read_env_options();
  const GemmPlan pl = gemm_plan(M, N, K, L, false, num_sms_of(dev), opt);
  g.prefetch = opt.prefetch;
  g.inject = opt.fault_inject;
  g.b_evict = opt.b_evict >= 0 ? opt.b_evict : pl.b_evict;
  rc = apply_plan("nvfp4_gemm", dev, pl, g, stream);
  if (rc) return rc;
  const char* why = nullptr;
  cudaError_t e = launch_gemm(g, num_sms_of(dev), static_cast<cudaStream_t>(stream), &why);
  if (e != cudaSuccess)
    return fail(NVFP4_ERR_CUDA, "nvfp4_gemm: %s", why ? why : cudaGetErrorString(e));
  return NVFP4_OK;
}

NVFP4_API int nvfp4_dual_gemm(const void* a, const void* b1, const void* b2, const void* sfa_blk, const void* sfb1_blk,
                    const void* sfb2_blk, void* c, int M, int N, int K, int L, int64_t a_lstride, int64_t b_lstride,
                    int64_t sfa_lstride, int64_t sfb_lstride, int64_t ldc, int64_t c_lstride, void* stream) {
  int rc = check_gemm_common("nvfp4_dual_gemm", a, b1, sfa_blk, sfb1_blk, c, M, N, K, L, a_lstride, b_lstride,
                             sfa_lstride, sfb_lstride, ldc, c_lstride);
  if (rc) return rc;
  if (!b2 || !sfb2_blk) return fail(NVFP4_ERR_NULL, "nvfp4_dual_gemm: null pointer");
  if (!aligned(b2, 16) || !aligned(sfb2_blk, 16))
    return fail(NVFP4_ERR_ALIGN, "nvfp4_dual_gemm: b2 and its scales need 16-byte alignment");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4_ERR_DEVICE, "nvfp4_dual_gemm: no CUDA device");
  GemmArgs g{};
  g.a = a;
  g.b = b1;
  g.b2 = b2;
  g.sfa = sfa_blk;
  g.sfb = sfb1_blk;
  g.sfb2 = sfb2_blk;
  g.c = c;
  g.M = M;
  g.N = N;
  g.K = K;
  g.L = L;
  g.a_lstride = a_lstride;
  g.b_lstride = b_lstride;
  g.b2_lstride = b_lstride;
  g.sfa_lstride = sfa_lstride;
  g.sfb_lstride = sfb_lstride;
  g.sfb2_lstride = sfb_lstride;
  g.ldc = ldc;
  g.c_lstride = c_lstride;
  g.status = status_ptr(dev);
  const EnvOptions opt = read_env_options();
  const GemmPlan pl = gemm_plan(M, N, K, L, true, num_sms_of(dev), opt);
  g.prefetch = opt.prefetch;
  g.inject = opt.fault_inject;
  g.b_evict = opt.b_evict >= 0 ? opt.b_evict : pl.b_evict;
  rc = apply_plan("nvfp4_dual_gemm", dev, pl, g, stream);
  if (rc) return rc;
  const char* why = nullptr;
  cudaError_t e = launch_dual_gemm(g, num_sms_of(dev), static_cast<cudaStream_t>(stream), &why);
  if (e != cudaSuccess)
    return fail(NVFP4_ERR_CUDA, "nvfp4_dual_gemm: %s", why ? why : cudaGetErrorString(e));
  return NVFP4_OK;
}


NVFP4_API int nvfp4_quantize(const void* x, int dtype, void* packed, void* sf_blk, int rows, int K, int L,
                             int64_t x_lstride, int64_t packed_lstride, int64_t sf_lstride, float global_scale,
                             void* stream) {
  if (!x || !packed || !sf_blk) return fail(NVFP4_ERR_NULL, "nvfp4_quantize: null pointer");
  if (dtype != 0 && dtype != 1) return fail(NVFP4_ERR_SHAPE, "nvfp4_quantize: dtype must be 0 (fp16) or 1 (bf16)");
  if (rows <= 0 || K <= 0 || L <= 0 || rows % 128 || K % 64)
    return fail(NVFP4_ERR_SHAPE, "nvfp4_quantize: rows=%d must be a multiple of 128 and K=%d of 64", rows, K);
  if (!(global_scale > 0.f)) return fail(NVFP4_ERR_SHAPE, "nvfp4_quantize: global_scale must be > 0");
  if (!aligned(x, 32) || !aligned(packed, 8) || !aligned(sf_blk, 4) || (x_lstride % 16) || (packed_lstride % 8) ||
      (sf_lstride % 4))
    return fail(NVFP4_ERR_ALIGN, "nvfp4_quantize: x needs 32-byte, packed 8-byte, scales 4-byte alignment");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4_ERR_DEVICE, "nvfp4_quantize: no CUDA device");
  QuantArgs a{x, dtype, packed, sf_blk, rows, K, L, x_lstride, packed_lstride, sf_lstride, global_scale};
  cudaError_t e = launch_quantize(a, num_sms_of(dev), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "nvfp4_quantize: %s", cudaGetErrorString(e));
  return NVFP4_OK;
}

static int scale_layout(const char* name, bool to_blocked, const void* src, void* dst, int rows, int sk, int L,
                        int64_t plain_row_stride, int64_t plain_lstride, int64_t blk_lstride, void* stream) {
  if (!src || !dst) return fail(NVFP4_ERR_NULL, "%s: null pointer", name);
  if (rows <= 0 || sk <= 0 || L <= 0 || rows % 128 || sk % 4)
    return fail(NVFP4_ERR_SHAPE, "%s: rows=%d must be a multiple of 128 and K/16=%d of 4", name, rows, sk);
  if (!aligned(src, 4) || !aligned(dst, 4) || (plain_row_stride % 4) || (plain_lstride % 4) || (blk_lstride % 4))
    return fail(NVFP4_ERR_ALIGN, "%s: bases and strides must be multiples of 4 bytes", name);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(NVFP4_ERR_DEVICE, "%s: no CUDA device", name);
  ScaleLayoutArgs a{src, dst, rows, sk, L, plain_row_stride, plain_lstride, blk_lstride};
  cudaError_t e = launch_scale_layout(a, to_blocked, num_sms_of(dev), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
  return NVFP4_OK;
}

NVFP4_API int nvfp4_scales_to_blocked(const void* plain, void* blk, int rows, int sk, int L, int64_t plain_row_stride,
                                      int64_t plain_lstride, int64_t blk_lstride, void* stream) {
  return scale_layout("nvfp4_scales_to_blocked", true, plain, blk, rows, sk, L, plain_row_stride, plain_lstride,
                      blk_lstride, stream);
}

NVFP4_API int nvfp4_scales_from_blocked(const void* blk, void* plain, int rows, int sk, int L,
                                        int64_t plain_row_stride, int64_t plain_lstride, int64_t blk_lstride,
                                        void* stream) {
  return scale_layout("nvfp4_scales_from_blocked", false, blk, plain, rows, sk, L, plain_row_stride, plain_lstride,
                      blk_lstride, stream);
}

// Packed-argument forms (include/nvfp4_b200.h): the same calls, one pointer.
NVFP4_API int nvfp4_gemv_call(const nvfp4_gemv_args* x) {
  if (!x) return fail(NVFP4_ERR_NULL, "nvfp4_gemv_call: null argument block");
  return nvfp4_gemv(x->a, x->b, x->sfa_blk, x->sfb_blk, x->c, x->M, x->K, x->L, x->a_lstride, x->b_lstride,
                    x->sfa_lstride, x->sfb_lstride, x->c_lstride, x->stream);
}

NVFP4_API int nvfp4_gemm_call(const nvfp4_gemm_args* x) {
  if (!x) return fail(NVFP4_ERR_NULL, "nvfp4_gemm_call: null argument block");
  return nvfp4_gemm(x->a, x->b, x->sfa_blk, x->sfb_blk, x->c, x->M, x->N, x->K, x->L, x->a_lstride, x->b_lstride,
                    x->sfa_lstride, x->sfb_lstride, x->ldc, x->c_lstride, x->stream);
}

NVFP4_API int nvfp4_dual_gemm_call(const nvfp4_gemm_args* x) {
  if (!x) return fail(NVFP4_ERR_NULL, "nvfp4_dual_gemm_call: null argument block");
  return nvfp4_dual_gemm(x->a, x->b, x->b2, x->sfa_blk, x->sfb_blk, x->sfb2_blk, x->c, x->M, x->N, x->K, x->L,
                         x->a_lstride, x->b_lstride, x->sfa_lstride, x->sfb_lstride, x->ldc, x->c_lstride, x->stream);
}
