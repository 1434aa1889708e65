/* cmpx.h -- C ABI of the B200 (sm_100a) dense matmul library libcmpx.so.
 *
 * Drop-in boundary for the dense matmul path of cmpext3 (eastmoe/cmp_ext).
 * The reference exposes three C++-linkage launchers that take row-major
 * device pointers with packed strides and launch on the legacy default
 * stream, returning nothing:
 *
 *   void launch_matmul_fp16(const void* A, const void* B, void* C, int M, int N, int K);
 *   void launch_matmul_fp32(const float* A, const float* B, float* C, int M, int N, int K);
 *   void launch_matmul_bf16(const void* A, const void* B, void* C, int M, int N, int K);
 *   void launch_add_bias_{fp16,fp32,bf16}(void* C, const void* bias, int rows, int cols);
 *   void launch_attention_{fp32,fp16,bf16}(q, k, v, output, int B, int H, int S, int D, float scale);
 *
 *   (reference src/main.cpp:12-19; definitions src/cuda/fp16_matmul.cu:301-366,
 *    src/cuda/fp32_matmul.cu:236-287, src/cuda/bf16_matmul.cu:232-317)
 *
 * libcmpx.so exports those six symbols unchanged (C++ linkage, same
 * signatures, same default-stream behaviour) so a binary linked against the
 * reference resolves against this library, plus the extern "C" entry points
 * below, which add an explicit stream, explicit strides, batching, a fused
 * bias and a status code.  Nothing in these signatures is a torch type.
 *
 * Semantics (all entry points): C[M,N] = A[M,K] * B[K,N] (+ bias[N]) with
 * row-major operands.  fp16 / bf16 inputs are multiplied on the tensor cores
 * with fp32 accumulation and rounded once to the output type.  fp32 inputs
 * use a 3xTF32 split-precision tensor-core kernel (hi*hi + hi*lo + lo*hi,
 * fp32 accumulation); shapes the TMA engine cannot describe (row strides that
 * are not a multiple of 16 bytes, unaligned base pointers) use a CUDA-core
 * kernel with fp32 FMA accumulation.
 *
 * All pointers are device pointers on the current device.  Calls are
 * asynchronous on `stream` (0 = legacy default stream).  Return value: 0 on
 * success, otherwise a cmpx_status code; nothing is launched on error.
 */
#ifndef CMPX_H_
#define CMPX_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CMPX_API __attribute__((visibility("default")))
#else
#define CMPX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* cmpx_stream_t; /* == cudaStream_t */

typedef enum {
  CMPX_OK = 0,
  CMPX_ERR_INVALID_ARG = 1, /* null pointer, negative size, stride too small, bad enum */
  CMPX_ERR_UNSUPPORTED = 2, /* forced path cannot handle this shape / alignment */
  CMPX_ERR_CUDA = 3,        /* a CUDA runtime/driver call or kernel launch failed */
  CMPX_ERR_NO_MEMORY = 4,   /* library-managed workspace could not be allocated */
  CMPX_ERR_DEVICE = 5,      /* a kernel reported a device-side error (bounded wait expired) */
  CMPX_ERR_WORKSPACE = 6,   /* caller workspace smaller than cmpx_gemm_workspace_size() */
  CMPX_ERR_TOO_LARGE = 7    /* problem exceeds the fixed scratch of cmpx_matmul_skinny_noalloc() */
} cmpx_status;

typedef enum { CMPX_F16 = 0, CMPX_BF16 = 1, CMPX_F32 = 2 } cmpx_dtype;

typedef enum {
  CMPX_B_KN = 0, /* B is [K, N] row-major (matmul / bmm operand, reference layout) */
  CMPX_B_NK = 1  /* B is [N, K] row-major (nn.Linear weight; no transpose copy) */
} cmpx_b_layout;

typedef enum {
  CMPX_PATH_AUTO = 0,
  CMPX_PATH_TC = 1,     /* tcgen05 persistent tile kernel (fp16/bf16) or 3xTF32 (fp32) */
  CMPX_PATH_SKINNY = 2, /* swap-AB stream-K tcgen05 kernel, M <= 128, fp16/bf16 */
  CMPX_PATH_SIMT = 3,   /* CUDA-core fallback */
  CMPX_PATH_BF16X3 = 4  /* fp32 only, opt-in: the tile kernel on bf16 hi/lo splits (hi*hi + hi*lo + lo*hi
                           on the bf16 tensor rate, twice the tf32 rate); normwise error ~5e-6 against
                           ~1e-6 for 3xTF32.  Needs K % 8 == 0.  AUTO never picks it; the environment
                           variable CMPX_FORCE_PATH=bf16x3 makes fp32 calls take it. */
} cmpx_path;

/* General batched GEMM descriptor.  Strides are in elements. */
typedef struct {
  int dtype;              /* cmpx_dtype, same for A, B, C, bias */
  const void* A;          /* [batch][M][K], row stride lda, batch stride stride_a */
  const void* B;          /* CMPX_B_KN: [batch][K][N] (ldb >= N); CMPX_B_NK: [batch][N][K] (ldb >= K) */
  void* C;                /* [batch][M][N], row stride ldc, batch stride stride_c */
  const void* bias;       /* optional [N] (NULL = none), fused into the epilogue */
  int64_t batch, M, N, K; /* all >= 0 */
  int64_t lda, ldb, ldc;
  int64_t stride_a, stride_b, stride_c;  /* stride_a == 0 with batch > 1: one A shared by every batch entry */
  int b_layout;           /* cmpx_b_layout */
  int path;               /* cmpx_path (AUTO unless a test forces one) */
  void* workspace;        /* optional caller scratch (device, 16-byte aligned, zero-filled before its
                             first use; calls leave its counters at zero); NULL = library-managed */
  size_t workspace_bytes;
  int bias_along_m;       /* 0: bias[N] added to every row; 1: bias[M] added to every column
                             (per output channel of a 1x1 convolution in NCHW) */
  void* const* peer_C;    /* optional: n_peer_C more outputs with C's layout (strides), e.g. the same
                             rows of C in peer GPUs' memory mapped into this process; the epilogue
                             stores every C element to C and to each of them (tile paths only) */
  int n_peer_C;           /* 0..7 */
  void* mc_C;             /* optional: NVLink multicast address with C's layout (the multicast mapping of
                             a buffer that C is part of, e.g. symmetric memory bound to a multicast
                             object on every GPU); the epilogue then stores each output element once,
                             through it, and the switch writes it into every bound buffer, C's included.
                             fp16/bf16, M > 128 (the CTA-pair kernel), N % 8 == 0, no peer_C; the
                             caller orders the other GPUs' use of their buffers. NULL = none */
} cmpx_gemm_args;

/* Replaces launch_matmul_fp16 (reference src/cuda/fp16_matmul.cu:301-340;
 * declared src/main.cpp:12).  Packed strides lda=K, ldb=ldc=N. */
CMPX_API int cmpx_matmul_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                    cmpx_stream_t stream);

/* Replaces launch_matmul_bf16 (reference src/cuda/bf16_matmul.cu:232-254;
 * declared src/main.cpp:14). */
CMPX_API int cmpx_matmul_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                     cmpx_stream_t stream);

/* Replaces launch_matmul_fp32 (reference src/cuda/fp32_matmul.cu:236-265;
 * declared src/main.cpp:13). */
CMPX_API int cmpx_matmul_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                    cmpx_stream_t stream);

/* Replaces the per-batch launch loop of custom_bmm_forward
 * (reference src/main.cpp:313-351) and the weight.t().contiguous() +
 * launch_matmul_* + launch_add_bias_* sequence of custom_linear_forward
 * (reference src/main.cpp:182-246) with one launch. */
CMPX_API int cmpx_gemm(const cmpx_gemm_args* args, cmpx_stream_t stream);

/* Scratch bytes cmpx_gemm needs for these args when the caller supplies the
 * workspace (0 when the chosen path needs none). */
CMPX_API size_t cmpx_gemm_workspace_size(const cmpx_gemm_args* args);

/* Which path cmpx_gemm would take (cmpx_path value; never AUTO), or -1 for
 * invalid args. */
CMPX_API int cmpx_gemm_select_path(const cmpx_gemm_args* args);

/* M-sharded GEMM with its output rows copied to peer GPUs while it runs.
 * No counterpart in the reference, which has no multi-GPU code; this is the
 * all-gather of C for the row-sharded layout of the matmul path (rank r
 * computes rows [r S, (r+1) S) of C, every rank wants the whole C).
 *
 * Computes `args` (fp16/bf16, batch 1, M > 128: the CTA-pair tile kernel)
 * into args->C on `stream`.  The kernel counts finished output tiles per
 * block -- an M group of its raster (8 pair-tile rows, 2048 rows; the
 * CMPX_TC_GROUP_M setting) times one of n_groups groups of 256-column tile
 * columns -- in `flags` (n_flags ints, zero before the first call; at least
 * ceil(ceil(M / 256) / 8) * n_groups of them, else CMPX_ERR_WORKSPACE).
 * copy_streams[p % n_copy_streams] waits on each block's flag (a stream
 * memory operation, no SM time) and copies the block to peer_C[p] (same
 * ldc) with cudaMemcpy2DAsync, i.e. on a copy engine over NVLink, while later
 * tiles are still computing.  `stream` waits for every copy before its next
 * work.  `epoch` is 1 on the first call with a given `flags` array and grows
 * by one per call (flags are never cleared).  peer_C entries must be mapped
 * into this process (peer access or a symmetric-memory mapping); the caller
 * orders the peers' use of their outputs (e.g. a barrier before and after).
 * n_peers = 0 runs the flagged GEMM alone.  CMPX_ERR_UNSUPPORTED when the
 * shape does not run the CTA-pair kernel. */
CMPX_API int cmpx_gemm_gather_ce(const cmpx_gemm_args* args, void* const* peer_C, int n_peers, int* flags,
                                 int n_flags, int n_groups, unsigned int epoch, cmpx_stream_t stream,
                                 const cmpx_stream_t* copy_streams, int n_copy_streams);

/* Replaces launch_add_bias_{fp16,fp32,bf16} (reference
 * src/cuda/fp16_matmul.cu:357-366, src/cuda/fp32_matmul.cu:272-287,
 * src/cuda/bf16_matmul.cu:308-317; declared src/main.cpp:17-19).
 * C[r, c] += bias[c] for every row, computed in fp32 and rounded once; unlike
 * the reference it is correct for odd (fp16) and non-multiple-of-4 (fp32)
 * column counts. */
CMPX_API int cmpx_add_bias(int dtype, void* C, const void* bias, int64_t rows, int64_t cols, cmpx_stream_t stream);

/* Skinny-M (decode) matmul that allocates no device memory.  No counterpart
 * in the reference, which allocates nothing itself because it has no
 * scratch at all.
 *
 * For callers that cannot call cudaMalloc: code that runs inside a fixed
 * memory budget handed out by a host framework, allocator hooks that must not
 * recurse into the allocator, or a process that sets the device up once and
 * may not allocate afterwards.  cmpx_gemm's skinny path needs ~2.7-20 MB of
 * scratch (fp32 partial sums of the split K range, plus per-tile counters)
 * and gets it from cudaMalloc or from a caller workspace; this variant uses
 * a fixed array compiled into libcmpx.so instead (about 10.8 MB, held on
 * every GPU that loads the library until the process exits).
 *
 * Computes C[M,N] = A[M,K] * B (+ bias[N]) for fp16/bf16 with packed
 * row-major operands: A [M,K]; B [K,N] (b_layout CMPX_B_KN) or [N,K]
 * (CMPX_B_NK); C [M,N]; same kernel and fp32 accumulation as cmpx_gemm's
 * skinny path, with one 128-column slab per work unit.  Limits: M <= 64,
 * ceil(N/128) <= 16384, at most 160 SMs on the device -- otherwise
 * CMPX_ERR_TOO_LARGE.  Pointers and row strides must be 16-byte aligned
 * (else CMPX_ERR_UNSUPPORTED).
 *
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  Every call on a device shares the one array:
 * calls that may overlap on the GPU (different streams, or different host
 * threads) race and must be serialised by the caller.  The per-tile counters
 * the kernel needs at zero are cleared (cudaMemsetAsync) on `stream` at the
 * start of every call. */
CMPX_API int cmpx_matmul_skinny_noalloc(int dtype, const void* A, const void* B, void* C, const void* bias,
                                        int64_t M, int64_t N, int64_t K, int b_layout, cmpx_stream_t stream);

/* Scaled dot-product attention O = softmax(scale * Q K^T) V.  Replaces
 * launch_attention_{fp32,fp16,bf16} (reference src/main.cpp:48-50;
 * src/cuda/fp16_attention.cu:158-186, src/cuda/bf16_attention.cu:97-104,
 * src/cuda/fp32_attention.cu:200-217), which libcmpx.so also exports under
 * their C++ names (legacy default stream, no status).
 *
 * Q, K, V, O: contiguous [B, H, S, D] device tensors of `dtype` (the same S
 * for queries and keys, as in the reference).  No mask.  fp16 / bf16 with
 * D = 64 or 128 and 16-byte aligned pointers run a tcgen05 flash-attention
 * kernel (QK^T and PV on the tensor cores, fp32 accumulation, online
 * softmax in fp32); other D up to 512 and fp32 run a CUDA-core kernel with
 * the same fp32 arithmetic.  path: CMPX_PATH_AUTO, CMPX_PATH_TC or
 * CMPX_PATH_SIMT (CMPX_ERR_UNSUPPORTED when the forced path cannot run the
 * shape). */
CMPX_API int cmpx_attention(int dtype, const void* Q, const void* K, const void* V, void* O, int64_t B, int64_t H,
                            int64_t S, int64_t D, float scale, int path, cmpx_stream_t stream);

/* Which attention path cmpx_attention would take (cmpx_path value), or -1. */
CMPX_API int cmpx_attention_select_path(int dtype, const void* Q, const void* K, const void* V, const void* O,
                                        int64_t D, int path);

/* Reads and clears the device-side error word of the current device
 * (synchronises the device).  *code receives the first error a kernel
 * recorded since the last call (0 = none).  When it is non-zero, the counter
 * region of the library-managed workspace is zeroed again (a launch that gave
 * up can leave counters behind); a caller workspace must then be re-zeroed by
 * the caller.  Returns CMPX_OK or CMPX_ERR_CUDA. */
CMPX_API int cmpx_device_error(int* code);

/* Diagnostic; no counterpart in the reference (which has no bounded waits).
 * Runs one kernel whose single wait -- the bounded mbarrier wait every
 * pipeline role of the GEMM kernels uses -- targets a barrier phase nothing
 * completes, with a limit of `timeout_ns` (1 ns .. 10 s).  The kernel records
 * an error code in the device error word and returns; the call synchronises
 * `stream` and returns CMPX_ERR_DEVICE when the wait expired as intended.
 * The device stays usable; read (and clear) the code with cmpx_device_error. */
CMPX_API int cmpx_selftest_bounded_wait(unsigned long long timeout_ns, cmpx_stream_t stream);

/* Human-readable name of a cmpx_status value. */
CMPX_API const char* cmpx_status_string(int status);

/* Library version, e.g. "cmpx 0.1.0 sm_100a". */
CMPX_API const char* cmpx_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* CMPX_H_ */
