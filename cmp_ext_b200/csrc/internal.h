// Internal interface between the C-ABI dispatcher (cmpx_api.cu) and the
// kernel translation units.  Not installed; not part of the public ABI.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/cmpx.h"

namespace cmpx {

// Extra copies of C to write besides C itself: peer GPUs' buffers (mapped
// into this process) with C's layout, so an M-sharded GEMM can deliver its
// rows to every rank from the epilogue.  Plain stores over NVLink.
constexpr int kMaxPeerOut = 7;
struct PeerOut {
  void* base[kMaxPeerOut];
  int n;
};

// TMA store maps of C and of its peer copies (box 32 x 32, no swizzle), for
// the CTA-pair kernel's staged epilogue: m[0] = C, m[1..n-1] = peers.
struct OutMaps {
  CUtensorMap m[1 + kMaxPeerOut];
  int n;
};

// A fully resolved batched GEMM: C[b] = A[b] * op(B[b]) (+ bias), row-major.
//   A    : [M, K] with row stride lda, batch stride sa (elements)
//   B    : b_kmajor == 0 -> [K, N] row-major (ldb >= N)   (matmul / bmm)
//          b_kmajor == 1 -> [N, K] row-major (ldb >= K)   (linear weight)
//   C    : [M, N] with row stride ldc, batch stride sc
//   bias : optional [N], same dtype as C
struct Gemm {
  int dtype;
  const void* A;
  const void* B;
  void* C;
  const void* bias;
  int64_t batch, M, N, K;
  int64_t lda, ldb, ldc;
  int64_t sa, sb, sc;
  int b_kmajor;
  int a_bcast;  // batch > 1 and stride_a == 0: every batch entry uses the same A
  int bias_m;   // bias has M entries (one per row) instead of N (one per column)
  PeerOut peers;  // also write C to these (same layout), n = 0: none
  // Multicast address (NVLink multicast object) of C's layout: the CTA-pair
  // kernel writes every output element once through it, reaching C and every
  // other buffer bound to the object; nullptr = none.
  void* mc_C = nullptr;
  // Progress flags (CTA-pair kernel only; nullptr = none): after its rows of
  // the output tile (tm, tn) are stored, each epilogue warp of the pair adds
  // 1 to col_flags[(tm / group_m) * column_groups + tn / flag_tiles]
  // (system-scope release; group_m = tc2_group_m(), the raster's M group),
  // so another stream can start on finished blocks while the GEMM runs.
  int* col_flags = nullptr;
  int flag_tiles = 0;
};

inline int elem_bytes(int dtype) { return dtype == CMPX_F32 ? 4 : 2; }

// Per-device facts cached by the dispatcher.
struct DeviceInfo {
  int num_sms;
  int max_smem_optin;
};

// Tensor-core main kernel (fp16 / bf16 inputs, fp32 TMEM accumulate).
// tA/tB are 3-D TMA maps over A and B (see cmpx_api.cu for box shapes).
cudaError_t launch_tc_f16(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tB, int bn,
                          const DeviceInfo& dev, int* dev_err, cudaStream_t s);

// CTA-pair (cta_group::2) variant of the fp16/bf16 tile kernel: 256 x pair_n
// output tiles (pair_n = 128 or 256).  tA box = {64, 128}; tB box = {64, 64}
// for a [K,N] B, {64, pair_n / 2} for an [N,K] B.
// ws: stream-K workspace of tc2_workspace_bytes() (shares the skinny
// path's layout: fixed zeroed counter region first), or nullptr to run
// whole tiles only.
size_t tc2_workspace_bytes(const Gemm& g, int pair_n, const DeviceInfo& dev);
// om: when non-null, the epilogue stages each 32 x 32 output chunk in shared
// memory and writes it with TMA stores to every map in om (used when the
// output also goes to peer GPUs: bulk writes instead of 16-byte stores).
cudaError_t launch_tc2_f16(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tB, int pair_n, void* ws,
                           const DeviceInfo& dev, int* dev_err, cudaStream_t s, const OutMaps* om = nullptr);

// 3xTF32 tensor-core kernel for fp32: tA/tA2 map the tf32 hi/lo splits of A,
// tB/tB2 those of B, both packed K-major (B as [N][K]).
cudaError_t launch_tc_tf32x3(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tA2, const CUtensorMap& tB,
                             const CUtensorMap& tB2, const DeviceInfo& dev, int* dev_err, cudaStream_t s);
// bf16x3 variant: the same maps over packed bf16 hi/lo splits (box {64, 128}),
// or with b_nmajor the splits of B kept [K][N] (box {64 of N, 64 of K}).
cudaError_t launch_tc_bf16x3(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tA2, const CUtensorMap& tB,
                             const CUtensorMap& tB2, bool b_nmajor, const DeviceInfo& dev, int* dev_err,
                             cudaStream_t s);

// Splits fp32 X [batch][rows][cols] (row stride ld, batch stride sx) into
// packed tf32 hi and lo parts: [batch][rows][cols] contiguous, or with
// transpose = true [batch][cols][rows] contiguous.
cudaError_t launch_split_tf32(const float* X, float* hi, float* lo, int64_t batch, int64_t rows, int64_t cols,
                              int64_t ld, int64_t sx, bool transpose, int num_sms, cudaStream_t s);
// The same with bf16 hi = rn(x), lo = rn(x - hi) (hi, lo: __nv_bfloat16).
cudaError_t launch_split_bf16(const float* X, void* hi, void* lo, int64_t batch, int64_t rows, int64_t cols,
                              int64_t ld, int64_t sx, bool transpose, int num_sms, cudaStream_t s);

// Swap-AB stream-K kernel for skinny M (M <= 128), fp16/bf16.
// tBop maps B as the MMA's 128-row operand, tAop maps A as the MMA's
// narrow operand (box rows = mn).  ws: fp32 partials, counters: per-tile ints
// that are zero on entry and left zero on exit.
constexpr int64_t kSkinnyMaxTiles = 16384;
constexpr size_t kSkinnyCounterBytes = size_t(kSkinnyMaxTiles) * 4 * sizeof(int);
size_t skinny_workspace_bytes(const Gemm& g, const DeviceInfo& dev);
size_t skinny_partials_bytes(const DeviceInfo& dev, int ns, int mn);
int skinny_mn(int64_t M);
int skinny_ns(const Gemm& g, const DeviceInfo& dev);
int64_t skinny_tiles(const Gemm& g, const DeviceInfo& dev);
cudaError_t launch_skinny(const Gemm& g, const CUtensorMap& tBop, const CUtensorMap& tAop, void* ws,
                          const DeviceInfo& dev, int* dev_err, cudaStream_t s);

// CUDA-core fallback for shapes the TMA paths cannot describe.
cudaError_t launch_simt(const Gemm& g, cudaStream_t s);

// C = bias (broadcast over rows) or 0, used when K == 0.
cudaError_t launch_fill_bias(const Gemm& g, cudaStream_t s);

// Stand-alone row-broadcast bias add (reference launch_add_bias_* semantics,
// computed in fp32 and rounded once).
cudaError_t launch_add_bias(int dtype, void* C, const void* bias, int64_t rows, int64_t cols, cudaStream_t s);

// cmpx_gemm for the CTA-pair kernel with column-progress flags (see
// Gemm::col_flags); CMPX_ERR_UNSUPPORTED for anything that would not run the
// 256-column pair-tile kernel on whole tiles.
int run_gemm_flagged(const cmpx_gemm_args* args, int* flags, int flag_tiles, cudaStream_t s);

// Device error word (see ptx.cuh DeviceError).
int* device_error_word();

// Facts and error word of the current device (initialising them once), and
// the TMA descriptor encoder the dispatcher uses; for entry points that live
// next to their kernels.
int device_facts(DeviceInfo* info, int** err_word);
int encode_tmap_3d(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t rows, uint64_t batch,
                   uint64_t ld, uint64_t bstride, uint32_t box_inner, uint32_t box_rows);

// Programmatic dependent launch for the GEMM kernels (on unless CMPX_PDL=0).
bool pdl_enabled();
// Sleep between polls of a tile kernel's epilogue while it waits for the
// next accumulator (CMPX_EPI_SLEEP_NS, default 0 = spin).
unsigned epilogue_sleep_ns();
// Pair tiles per M group of the CTA-pair kernel's raster (CMPX_TC_GROUP_M,
// default 8): the tiles of one group share A rows and walk B's columns.
int tc2_group_m();
// Tile width of the 3xTF32 kernel: 256 (128 x 256 tiles, two stages) unless
// CMPX_TF32_BN=128 (128 x 128 tiles, three stages).
int tf32x3_block_n();
// Fills `attr` (one slot) and cfg.attrs / cfg.numAttrs for a PDL launch, or
// leaves cfg without attributes when PDL is off.
inline void apply_pdl(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, int used) {
  cfg.attrs = attr;
  cfg.numAttrs = used;
  if (pdl_enabled()) {
    attr[used].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[used].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = used + 1;
  }
}

}  // namespace cmpx

namespace cmpx {
// Sets a kernel's dynamic shared-memory limit once per device (the attribute
// is per function and device; setting it on every launch costs host time that
// shows up in short kernels' latency).  `done` must be a flag word owned by
// that one kernel (a static in its launcher): bit d = set on device d.
template <typename KernelPtr>
cudaError_t set_smem_once(KernelPtr kern, int bytes, unsigned long long& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit != 0) __atomic_fetch_or(&done, bit, __ATOMIC_RELEASE);
  return e;
}
}  // namespace cmpx
