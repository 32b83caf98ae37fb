/* C ABI of libnvfp4_b200.so — B200 (sm_100a) NVFP4 block-scaled GEMV, GEMM and
 * dual GEMM with a fused SiLU gate.
 *
 * These entry points replace the device work behind the reference's plugin
 * boundary `custom_kernel(data) -> output` of the three problems under
 * problems/nvidia/ (SwayamInSync/reference-kernels):
 *
 *   nvfp4_gemv       <- problems/nvidia/nvfp4_gemv/submission.py:28-54
 *                       (torch._scaled_mm per batch, column 0 kept) and
 *                       problems/nvidia/nvfp4_gemv/template_cute.py:199-247
 *   nvfp4_gemm       <- problems/nvidia/nvfp4_gemm/submission.py:708-761
 *                       (CuTe-DSL tcgen05 kernel launch)
 *   nvfp4_dual_gemm  <- problems/nvidia/nvfp4_dual_gemm/submission.py:894-957
 *
 * Data layouts are the reference's input_t tensors (task.py of each problem),
 * passed as raw device pointers: every operand is a stack of L contiguous
 * batch slices, slice l starting at base + l * <x>_lstride.
 *   packed e2m1 A/B : rows x K/2 bytes, two codes per byte, even K index in
 *                     the low nibble (torch.float4_e2m1fn_x2)
 *   plain scales    : rows x K/16 e4m3fn bytes, row-major (tuple slots 2-3)
 *   blocked scales  : the 128x4-blocked order of to_blocked
 *                     (nvfp4_gemm/reference.py:12-24), i.e. the memory order of
 *                     the "permuted" tuple slots: byte (i, j) at
 *                     (i/128)*(K/64)*512 + (j/4)*512 + (i%32)*16 + ((i%128)/32)*4 + j%4
 *   C               : fp16, row m of slice l at c + l*c_lstride + m*ldc
 *
 * All calls are asynchronous on `stream` (a cudaStream_t; NULL = legacy
 * default stream).  The tensor-core GEMV (always) and the GEMMs (when the
 * planner uses stream-K: more tiles than SMs or SM pairs, in an uneven last
 * wave, e.g. 1024x7168x16384) use a per-device workspace, which the library
 * allocates on the first call that needs it (a call that would have to grow
 * it inside a stream capture returns NVFP4_ERR_CUDA and enqueues nothing).  Every entry point returns 0 on
 * success or one of the NVFP4_ERR_* codes; nvfp4_last_error() then returns a
 * message (thread-local).  Nothing runs on the CPU: there is no fallback.
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  NVFP4_OK = 0,
  NVFP4_ERR_SHAPE = 1,  /* unsupported size (see each function) */
  NVFP4_ERR_ALIGN = 2,  /* pointer or stride alignment */
  NVFP4_ERR_NULL = 3,   /* null pointer */
  NVFP4_ERR_CUDA = 4,   /* launch / driver error (message has the CUDA string) */
  NVFP4_ERR_DEVICE = 5, /* no current CUDA device */
};

/* Message for the last non-zero return on this thread. */
const char* nvfp4_last_error(void);

/* ABI revision of this header (2: adds the packed-argument *_call forms). */
int nvfp4_abi_version(void);

/* Reads (and optionally clears) the current device's status word, which the
 * tensor-core kernels set when a bounded pipeline wait runs out (non-zero;
 * 0 = ok).  Synchronous.  Returns -1 on a CUDA error.  Clearing a non-zero
 * status also zeroes the library's device workspaces (arrival counters,
 * stream-K flags, partial sums) on that device, which a kernel that gave up
 * may have left dirty, so the next call starts clean. */
int nvfp4_device_status(int clear);

/* Batched GEMV: c[m, l] = fp16( sum_k a[m,k,l]*sfa[m,k/16,l] * b[0,k,l]*sfb[0,k/16,l] ).
 * Replaces the reference GEMV custom_kernel (nvfp4_gemv/submission.py:28-54;
 * template_cute.py:199-247 reads the same blocked scales).
 *   a       : packed [L][M][K/2]            a_lstride   (bytes, multiple of 16)
 *   b       : packed [L][rows>=1][K/2]      b_lstride   (bytes; the reference pads b to 128 rows, row 0 is used)
 *   sfa_blk : blocked scales of A           sfa_lstride (bytes, = M*K/16 for the reference tensors)
 *   sfb_blk : blocked scales of b           sfb_lstride (bytes; 128-row block 0 is used)
 *   c       : fp16 [L][M]                   c_lstride   (elements)
 * Requires M % 128 == 0 and K % 64 == 0 (the reference's task.yml).  With
 * K % 256 == 0 it runs the TMA + tensor-core kernel, which splits row blocks
 * across SMs and uses a per-device workspace that the library allocates on the
 * first call that needs it; GEMV calls on one device must not overlap on the
 * GPU.  Other K use the SIMT kernel, which needs no workspace. */
int nvfp4_gemv(const void* a, const void* b, const void* sfa_blk, const void* sfb_blk, void* c, int M, int K, int L,
               int64_t a_lstride, int64_t b_lstride, int64_t sfa_lstride, int64_t sfb_lstride, int64_t c_lstride,
               void* stream);

/* nvfp4_gemv without any allocation.  No counterpart in the reference: it
 * exists for callers that cannot allocate device memory when they call the
 * GEMV -- for example code whose memory is fully reserved up front by a pool
 * or arena, or host code with no access to cudaMalloc -- and so cannot use
 * nvfp4_gemv, whose tensor-core path allocates a workspace on first use.
 * Same arguments, layouts and result as nvfp4_gemv; it runs the same
 * tensor-core kernel with its scratch memory (arrival counters and partial
 * sums) in a fixed array of NVFP4_GEMV_NOALLOC_SCRATCH_BYTES that the library
 * holds on every GPU that loads it until the process exits.
 *   - Requires M % 128 == 0 and K % 256 == 0; a shape whose scratch need
 *     exceeds the array is rejected with NVFP4_ERR_SHAPE and a message.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current and zeroes the
 *     arrival counters synchronously; make that first call before any
 *     stream capture.  The address is kept for the life of the process, so
 *     do not call it after cudaDeviceReset.
 *   - It calls no cudaMalloc / cudaFree.  Later calls only launch the
 *     kernel, which returns every counter it used to zero.
 *   - A bounded-wait timeout is recorded in the device status word like the
 *     other entry points'; nvfp4_device_status(1) then also re-zeroes the
 *     counters.
 *   - All calls share the one array, which keeps the last call's contents:
 *     calls that overlap on the GPU (other streams, other threads) race and
 *     give wrong results. */
#define NVFP4_GEMV_NOALLOC_SCRATCH_BYTES (4u << 20)
int nvfp4_gemv_noalloc(const void* a, const void* b, const void* sfa_blk, const void* sfb_blk, void* c, int M, int K,
                       int L, int64_t a_lstride, int64_t b_lstride, int64_t sfa_lstride, int64_t sfb_lstride,
                       int64_t c_lstride, void* stream);

/* Batched block-scaled GEMM: C = (A*sfA) (B*sfB)^T, fp32 accumulation, fp16 out.
 * Replaces nvfp4_gemm/submission.py:708-761.
 *   a       : packed [L][M][K/2]    a_lstride   (bytes)
 *   b       : packed [L][N][K/2]    b_lstride   (bytes)
 *   sfa_blk : blocked scales of A   sfa_lstride (bytes, = M*K/16 for the reference tensors)
 *   sfb_blk : blocked scales of B   sfb_lstride (bytes)
 *   c       : fp16 [L][M][ldc]      ldc, c_lstride (elements)
 * Requires M % 128 == 0, N % 128 == 0, K % 64 == 0 (the blocked scale layout;
 * K % 256 != 0 runs a partial last K tile),
 * 16-byte aligned bases and batch strides.  An N-shard of a larger problem is
 * passed as b + n0*K/2, sfb_blk + (n0/128)*K*8, c + n0 with ldc = full N. */
int nvfp4_gemm(const void* a, const void* b, const void* sfa_blk, const void* sfb_blk, void* c, int M, int N, int K,
               int L, int64_t a_lstride, int64_t b_lstride, int64_t sfa_lstride, int64_t sfb_lstride, int64_t ldc,
               int64_t c_lstride, void* stream);

/* Dual GEMM with fused gate: C = fp16( silu(A.B1^T) * (A.B2^T) ), both products
 * in fp32.  Replaces nvfp4_dual_gemm/submission.py:894-957.  Same layouts and
 * requirements as nvfp4_gemm; B1 and B2 share b_lstride / sfb_lstride. */
int nvfp4_dual_gemm(const void* a, const void* b1, const void* b2, const void* sfa_blk, const void* sfb1_blk,
                    const void* sfb2_blk, void* c, int M, int N, int K, int L, int64_t a_lstride, int64_t b_lstride,
                    int64_t sfa_lstride, int64_t sfb_lstride, int64_t ldc, int64_t c_lstride, void* stream);

/* NVFP4 quantiser: fp16 (dtype 0) or bf16 (dtype 1) x [L][rows][K] ->
 * packed e2m1 [L][rows][K/2] + e4m3 scales in the blocked layout, per
 * 16-element block: s = e4m3_rn_satfinite(amax / (6 * global_scale)),
 * q = e2m1_rn_satfinite(x / (s * global_scale)) (q = 0 where s == 0), so that
 * x ~= q * s * global_scale.  Produces the tensors generate_input builds
 * (nvfp4_gemm/reference.py:56-158, the permuted scale slots via to_blocked,
 * reference.py:12-24) from real data.  rows % 128 == 0, K % 64 == 0;
 * x_lstride in elements, packed_lstride / sf_lstride in bytes. */
int nvfp4_quantize(const void* x, int dtype, void* packed, void* sf_blk, int rows, int K, int L, int64_t x_lstride,
                   int64_t packed_lstride, int64_t sf_lstride, float global_scale, void* stream);

/* Scale layout conversion between the plain [L][rows][K/16] e4m3 layout
 * (row stride plain_row_stride bytes) and the 128x4-blocked layout of
 * to_blocked (nvfp4_gemm/reference.py:12-24); rows % 128 == 0, sk = K/16 with
 * sk % 4 == 0.  Pure byte permutations. */
int nvfp4_scales_to_blocked(const void* plain, void* blk, int rows, int sk, int L, int64_t plain_row_stride,
                            int64_t plain_lstride, int64_t blk_lstride, void* stream);
int nvfp4_scales_from_blocked(const void* blk, void* plain, int rows, int sk, int L, int64_t plain_row_stride,
                              int64_t plain_lstride, int64_t blk_lstride, void* stream);

/* Packed-argument forms of nvfp4_gemv / nvfp4_gemm / nvfp4_dual_gemm: the
 * same arguments in one struct, the same behaviour and return codes.  For
 * bindings whose per-argument conversion is costly (Python ctypes: ~2 us for
 * the 16-argument scalar form, ~0.5 us for one struct pointer), the caller can
 * keep one struct per input set and update only `stream` between calls. */
typedef struct {
  const void* a;
  const void* b;
  const void* sfa_blk;
  const void* sfb_blk;
  void* c;
  int32_t M, K, L, reserved;
  int64_t a_lstride, b_lstride, sfa_lstride, sfb_lstride, c_lstride;
  void* stream;
} nvfp4_gemv_args;

typedef struct {
  const void* a;
  const void* b;        /* B (nvfp4_gemm_call) or B1 (nvfp4_dual_gemm_call) */
  const void* b2;       /* B2; ignored by nvfp4_gemm_call */
  const void* sfa_blk;
  const void* sfb_blk;  /* blocked scales of B / B1 */
  const void* sfb2_blk; /* blocked scales of B2; ignored by nvfp4_gemm_call */
  void* c;
  int32_t M, N, K, L;
  int64_t a_lstride, b_lstride, sfa_lstride, sfb_lstride, ldc, c_lstride;
  void* stream;
} nvfp4_gemm_args;

int nvfp4_gemv_call(const nvfp4_gemv_args* args);
int nvfp4_gemm_call(const nvfp4_gemm_args* args);
int nvfp4_dual_gemm_call(const nvfp4_gemm_args* args);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_B200_H */
