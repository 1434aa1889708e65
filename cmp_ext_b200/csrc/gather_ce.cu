// M-sharded GEMM whose output rows reach every peer GPU through the copy
// engines while the GEMM is still running (the all-gather of C overlapped
// with the compute, without taking SMs from it).
//
// The reference has no multi-GPU code; this serves the row-sharded layout
// of the matmul path: rank r computes rows [r S, (r+1) S) of C and every
// rank wants the whole C.  The CTA-pair GEMM counts finished output tiles
// per block -- an M group of its raster (group_m pair-tile rows, which it
// sweeps column by column) times a group of pair-tile columns -- in device
// flags (gemm_tc2.cu, col_flags).  One copy stream per peer waits on each
// block's flag with a stream memory operation (cuStreamWaitValue32, GEQ),
// in the order the GEMM finishes them, and then copies the block into the
// peer's output with one 2-D cudaMemcpyAsync over NVLink.  Flags are never
// reset: call e (1, 2, ...) waits for e times a block's per-call count, so
// back-to-back calls need no clearing launch.
#include <cstring>
#include <mutex>

#include "internal.h"

namespace cmpx {
namespace {

typedef CUresult (*WaitValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
WaitValue32Fn g_wait32 = nullptr;
std::once_flag g_wait32_once;

int wait32_fn(WaitValue32Fn* out) {
  std::call_once(g_wait32_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWaitValue32", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_wait32 = reinterpret_cast<WaitValue32Fn>(fn);
  });
  *out = g_wait32;
  return g_wait32 != nullptr ? CMPX_OK : CMPX_ERR_CUDA;
}

}  // namespace
}  // namespace cmpx

using namespace cmpx;

extern "C" int cmpx_gemm_gather_ce(const cmpx_gemm_args* args, void* const* peer_C, int n_peers, int* flags,
                                   int n_flags, int n_groups, unsigned int epoch, cmpx_stream_t stream,
                                   const cmpx_stream_t* copy_streams, int n_copy_streams) {
  if (args == nullptr || n_peers < 0 || n_peers > kMaxPeerOut || flags == nullptr || n_groups < 1 || epoch == 0)
    return CMPX_ERR_INVALID_ARG;
  if (n_peers > 0 && (peer_C == nullptr || copy_streams == nullptr || n_copy_streams < 1))
    return CMPX_ERR_INVALID_ARG;
  for (int i = 0; i < n_peers; ++i)
    if (peer_C[i] == nullptr) return CMPX_ERR_INVALID_ARG;
  if (args->dtype != CMPX_F16 && args->dtype != CMPX_BF16) return CMPX_ERR_UNSUPPORTED;
  if (args->batch != 1 || args->n_peer_C != 0 || args->M <= 128 || args->K == 0) return CMPX_ERR_UNSUPPORTED;
  if (args->path != CMPX_PATH_AUTO && args->path != CMPX_PATH_TC) return CMPX_ERR_UNSUPPORTED;
  WaitValue32Fn wait32 = nullptr;
  int st = wait32_fn(&wait32);
  if (st != CMPX_OK) return st;

  // The GEMM (the CTA-pair kernel: M > 128, 256-column pair tiles), with
  // the column-progress flags.
  const int64_t pair_n = 256;
  const int64_t tiles_m = (args->M + 255) / 256;
  const int64_t tiles_n = (args->N + pair_n - 1) / pair_n;
  const int64_t flag_tiles = (tiles_n + n_groups - 1) / n_groups;
  const int64_t groups = (tiles_n + flag_tiles - 1) / flag_tiles;
  const int64_t group_m = tc2_group_m();
  const int64_t mgroups = (tiles_m + group_m - 1) / group_m;
  if (int64_t(n_flags) < mgroups * groups) return CMPX_ERR_WORKSPACE;
  cudaEvent_t ev_start = nullptr;
  if (n_peers > 0) {
    // the copies follow all earlier work on `stream` (e.g. the barrier that
    // frees the peers' outputs)
    if (cudaEventCreateWithFlags(&ev_start, cudaEventDisableTiming) != cudaSuccess) return CMPX_ERR_CUDA;
    if (cudaEventRecord(ev_start, stream) != cudaSuccess) return CMPX_ERR_CUDA;
  }
  st = run_gemm_flagged(args, flags, int(flag_tiles), stream);
  if (st != CMPX_OK) {
    if (ev_start) cudaEventDestroy(ev_start);
    return st;
  }
  if (n_peers == 0) return CMPX_OK;

  const int64_t E = 2;
  const int ns = n_copy_streams < n_peers ? n_copy_streams : n_peers;
  for (int c = 0; c < ns; ++c)
    if (cudaStreamWaitEvent(copy_streams[c], ev_start, 0) != cudaSuccess) return CMPX_ERR_CUDA;
  cudaEventDestroy(ev_start);
  const char* src = static_cast<const char*>(args->C);
  for (int64_t mg = 0; mg < mgroups; ++mg) {
    const int64_t row0 = mg * group_m * 256;
    const int64_t row1 = (mg + 1) * group_m * 256 < args->M ? (mg + 1) * group_m * 256 : args->M;
    const int64_t mtiles = (row1 - row0 + 255) / 256;
    for (int64_t j = 0; j < groups; ++j) {
      const int64_t col0 = j * flag_tiles * pair_n;
      const int64_t col1 = (j + 1) * flag_tiles * pair_n < args->N ? (j + 1) * flag_tiles * pair_n : args->N;
      const int64_t ntiles = (col1 - col0 + pair_n - 1) / pair_n;
      // 8 arrivals per pair tile (4 epilogue warps x 2 CTAs), per call
      const uint32_t target = uint32_t(uint64_t(epoch) * uint64_t(mtiles * ntiles * 8));
      int* flag = flags + mg * groups + j;
      for (int c = 0; c < ns; ++c) {
        if (wait32(reinterpret_cast<CUstream>(copy_streams[c]), reinterpret_cast<CUdeviceptr>(flag), target,
                   CU_STREAM_WAIT_VALUE_GEQ) != CUDA_SUCCESS)
          return CMPX_ERR_CUDA;
      }
      for (int p = 0; p < n_peers; ++p) {
        char* dst = static_cast<char*>(peer_C[p]);
        const size_t off = size_t(row0 * args->ldc + col0) * E;
        if (cudaMemcpy2DAsync(dst + off, size_t(args->ldc * E), src + off, size_t(args->ldc * E),
                              size_t((col1 - col0) * E), size_t(row1 - row0), cudaMemcpyDefault,
                              copy_streams[p % ns]) != cudaSuccess)
          return CMPX_ERR_CUDA;
      }
    }
  }
  // `stream` continues once every copy has landed
  for (int c = 0; c < ns; ++c) {
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return CMPX_ERR_CUDA;
    if (cudaEventRecord(ev, copy_streams[c]) != cudaSuccess || cudaStreamWaitEvent(stream, ev, 0) != cudaSuccess) {
      cudaEventDestroy(ev);
      return CMPX_ERR_CUDA;
    }
    cudaEventDestroy(ev);
  }
  return CMPX_OK;
}
