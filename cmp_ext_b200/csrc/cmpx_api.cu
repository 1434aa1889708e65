// C-ABI entry points of libcmpx.so: argument checks, path selection, TMA
// descriptor construction, workspace management, and the reference-compatible
// launch_matmul_* / launch_add_bias_* symbols.
//
// Reference boundary being replaced: the C++ launchers declared at
// src/main.cpp:12-19 and defined in src/cuda/{fp16,fp32,bf16}_matmul.cu.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>

#include "internal.h"

namespace cmpx {

__device__ int g_device_error = 0;

namespace {

constexpr int kMaxDevices = 64;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Library-managed device memory, per device, grow-only:
//   slot 0  scratch: fp32 hi/lo splits of the 3xTF32 path (contents do not
//           survive between calls)
//   slot 1  skinny-path workspace: fp32 partials plus per-tile counters that
//           must be zero on entry; the kernel leaves them zero, and no other
//           path writes this slot
struct DeviceState {
  bool init = false;
  int status = CMPX_OK;
  DeviceInfo info{};
  int* err_word = nullptr;
  std::mutex ws_mu;
  void* ws[2] = {nullptr, nullptr};
  size_t ws_bytes[2] = {0, 0};
};

DeviceState g_dev[kMaxDevices];
std::mutex g_init_mu;
EncodeTiledFn g_encode = nullptr;

int cuda_status(cudaError_t e) { return e == cudaSuccess ? CMPX_OK : CMPX_ERR_CUDA; }

// Resolves (once) the per-device facts and the driver's tensor-map encoder.
int device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CMPX_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return CMPX_ERR_UNSUPPORTED;
  DeviceState& d = g_dev[dev];
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (!d.init) {
    d.init = true;
    d.status = CMPX_OK;
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.info.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.info.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess) {
      d.status = CMPX_ERR_CUDA;
    } else if (major != 10 || minor != 0) {
      d.status = CMPX_ERR_UNSUPPORTED;  // kernels are built for sm_100a only
    } else if (cudaGetSymbolAddress(reinterpret_cast<void**>(&d.err_word), g_device_error) != cudaSuccess) {
      d.status = CMPX_ERR_CUDA;
    }
    if (d.status == CMPX_OK && g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr) {
        d.status = CMPX_ERR_CUDA;
      } else {
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
      }
    }
  }
  *out = &d;
  return d.status;
}

// Grow-only library-managed workspace slot, zero-filled when (re)allocated.
// A slot is shared by every call on the device: concurrent calls on
// different streams that need scratch must pass their own workspace.
int library_workspace(DeviceState& d, int slot, size_t bytes, void** out) {
  std::lock_guard<std::mutex> lk(d.ws_mu);
  if (d.ws_bytes[slot] < bytes) {
    if (d.ws[slot] != nullptr) {
      cudaDeviceSynchronize();  // earlier launches may still use the old buffer
      cudaFree(d.ws[slot]);
      d.ws[slot] = nullptr;
      d.ws_bytes[slot] = 0;
    }
    const size_t want = bytes + bytes / 4;
    if (cudaMalloc(&d.ws[slot], want) != cudaSuccess) {
      cudaGetLastError();
      return CMPX_ERR_NO_MEMORY;
    }
    if (cudaMemset(d.ws[slot], 0, want) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
      return CMPX_ERR_CUDA;
    d.ws_bytes[slot] = want;
  }
  *out = d.ws[slot];
  return CMPX_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3-D tiled map {inner, rows, batch}, 128-byte swizzle.
int encode_3d(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t rows, uint64_t batch,
              uint64_t ld, uint64_t bstride, uint32_t box_inner, uint32_t box_rows) {
  const uint64_t E = uint64_t(elem_bytes(dtype));
  if (batch <= 1 || bstride == 0) bstride = rows * ld;
  if (batch < 1) batch = 1;
  const CUtensorMapDataType dt = dtype == CMPX_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : dtype == CMPX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[3] = {inner, rows, batch};
  cuuint64_t strides[2] = {ld * E, bstride * E};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CMPX_OK : CMPX_ERR_CUDA;
}

// 3-D store map over C-shaped memory at `base`: {N, M, batch}, box 32 x 32,
// no swizzle (the CTA-pair kernel's staged epilogue).
int encode_out_map(CUtensorMap* m, const Gemm& g, void* base) {
  const uint64_t E = uint64_t(elem_bytes(g.dtype));
  const CUtensorMapDataType dt = g.dtype == CMPX_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t batch = g.batch < 1 ? 1 : uint64_t(g.batch);
  const uint64_t bstride = batch > 1 ? uint64_t(g.sc) : uint64_t(g.M) * uint64_t(g.ldc);
  cuuint64_t dims[3] = {uint64_t(g.N), uint64_t(g.M), batch};
  cuuint64_t strides[2] = {uint64_t(g.ldc) * E, bstride * E};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, dt, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CMPX_OK : CMPX_ERR_CUDA;
}

int env_forced_path() {
  static int forced = -1;
  if (forced < 0) {
    const char* e = std::getenv("CMPX_FORCE_PATH");
    forced = CMPX_PATH_AUTO;
    if (e != nullptr) {
      if (!std::strcmp(e, "tc")) forced = CMPX_PATH_TC;
      else if (!std::strcmp(e, "skinny")) forced = CMPX_PATH_SKINNY;
      else if (!std::strcmp(e, "simt")) forced = CMPX_PATH_SIMT;
      else if (!std::strcmp(e, "bf16x3")) forced = CMPX_PATH_BF16X3;
    }
  }
  return forced;
}

int validate(const cmpx_gemm_args* a) {
  if (a == nullptr) return CMPX_ERR_INVALID_ARG;
  if (a->dtype != CMPX_F16 && a->dtype != CMPX_BF16 && a->dtype != CMPX_F32) return CMPX_ERR_INVALID_ARG;
  if (a->b_layout != CMPX_B_KN && a->b_layout != CMPX_B_NK) return CMPX_ERR_INVALID_ARG;
  if (a->path < CMPX_PATH_AUTO || a->path > CMPX_PATH_BF16X3) return CMPX_ERR_INVALID_ARG;
  if (a->batch < 0 || a->M < 0 || a->N < 0 || a->K < 0) return CMPX_ERR_INVALID_ARG;
  const int64_t lim = (int64_t(1) << 31) - 1;
  if (a->M > lim || a->N > lim || a->K > lim) return CMPX_ERR_UNSUPPORTED;
  if (a->batch == 0 || a->M == 0 || a->N == 0) return CMPX_OK;
  if (a->C == nullptr) return CMPX_ERR_INVALID_ARG;
  if (a->ldc < a->N) return CMPX_ERR_INVALID_ARG;
  if (a->K > 0) {
    if (a->A == nullptr || a->B == nullptr) return CMPX_ERR_INVALID_ARG;
    if (a->lda < a->K) return CMPX_ERR_INVALID_ARG;
    if (a->ldb < (a->b_layout == CMPX_B_KN ? a->N : a->K)) return CMPX_ERR_INVALID_ARG;
  }
  if (a->stride_a < 0 || a->stride_b < 0 || a->stride_c < 0) return CMPX_ERR_INVALID_ARG;
  if (a->n_peer_C < 0 || a->n_peer_C > kMaxPeerOut) return CMPX_ERR_INVALID_ARG;
  if (a->mc_C != nullptr && a->n_peer_C > 0) return CMPX_ERR_INVALID_ARG;
  if (a->n_peer_C > 0) {
    if (a->peer_C == nullptr) return CMPX_ERR_INVALID_ARG;
    for (int i = 0; i < a->n_peer_C; ++i)
      if (a->peer_C[i] == nullptr) return CMPX_ERR_INVALID_ARG;
  }
  return CMPX_OK;
}

Gemm to_gemm(const cmpx_gemm_args* a) {
  Gemm g;
  g.dtype = a->dtype;
  g.A = a->A;
  g.B = a->B;
  g.C = a->C;
  g.bias = a->bias;
  g.batch = a->batch;
  g.M = a->M;
  g.N = a->N;
  g.K = a->K;
  g.lda = a->lda;
  g.ldb = a->ldb;
  g.ldc = a->ldc;
  g.sa = a->batch > 1 ? a->stride_a : a->M * a->lda;
  g.sb = a->batch > 1 ? a->stride_b : (a->b_layout == CMPX_B_KN ? a->K * a->ldb : a->N * a->ldb);
  g.sc = a->batch > 1 ? a->stride_c : a->M * a->ldc;
  g.b_kmajor = a->b_layout == CMPX_B_NK ? 1 : 0;
  g.a_bcast = (a->batch > 1 && a->stride_a == 0) ? 1 : 0;
  g.bias_m = a->bias_along_m ? 1 : 0;
  g.peers.n = a->n_peer_C;
  g.mc_C = a->mc_C;
  for (int i = 0; i < kMaxPeerOut; ++i) g.peers.base[i] = i < a->n_peer_C ? a->peer_C[i] : nullptr;
  return g;
}

// Can the TMA engine describe A and B as given (fp16/bf16) and can the
// epilogue use 16-byte stores on C?
bool tma_ok_16bit(const Gemm& g) {
  const int64_t E = 2;
  auto ok = [&](const void* p, int64_t ld, int64_t bs) {
    return aligned16(p) && (ld * E) % 16 == 0 && (g.batch <= 1 || (bs * E) % 16 == 0);
  };
  return ok(g.A, g.lda, g.sa) && ok(g.B, g.ldb, g.sb) && ok(g.C, g.ldc, g.sc);
}

// fp32 3xTF32: operands are re-packed K-major by the split pre-pass, so only
// the packed row length K and C need 16-byte alignment.
bool tma_ok_f32(const Gemm& g) {
  const bool a_ok = (g.K * 4) % 16 == 0;
  // B is re-packed K-major ([N][K]) by the split pre-pass; a [K,N] source is
  // transposed on the way by a float4 kernel (N, ldb multiples of 4, aligned).
  const bool b_ok = a_ok && (g.b_kmajor || (g.N % 4 == 0 && g.ldb % 4 == 0 && aligned16(g.B) &&
                                            (g.batch <= 1 || g.sb % 4 == 0)));
  const bool c_ok = aligned16(g.C) && (g.ldc * 4) % 16 == 0 && (g.batch <= 1 || (g.sc * 4) % 16 == 0);
  return a_ok && b_ok && c_ok;
}

// fp32 bf16x3: the same re-packing with 2-byte elements, so the packed row
// length K must be a multiple of 8.
bool tma_ok_bf16x3(const Gemm& g) { return g.K % 8 == 0 && tma_ok_f32(g); }

int choose_path(const Gemm& g, int requested, const DeviceInfo* dev) {
  int forced = requested != CMPX_PATH_AUTO ? requested : env_forced_path();
  if (g.K == 0) return CMPX_PATH_SIMT;  // fill kernel
  if (g.dtype == CMPX_F32) {
    const bool ok = tma_ok_f32(g);
    if (forced == CMPX_PATH_SKINNY) return -1;
    if (forced == CMPX_PATH_TC) return ok ? CMPX_PATH_TC : -1;
    if (forced == CMPX_PATH_BF16X3) return tma_ok_bf16x3(g) ? CMPX_PATH_BF16X3 : -1;
    if (forced == CMPX_PATH_SIMT) return CMPX_PATH_SIMT;
    const double work = double(g.batch) * double(g.M) * double(g.N) * double(g.K);
    return (ok && work >= double(1 << 22)) ? CMPX_PATH_TC : CMPX_PATH_SIMT;
  }
  const bool ok = tma_ok_16bit(g);
  if (forced == CMPX_PATH_BF16X3) {
    if (requested == CMPX_PATH_BF16X3) return -1;  // an fp32-only path
    forced = CMPX_PATH_AUTO;                       // the environment switch concerns fp32 only
  }
  if (forced == CMPX_PATH_TC) return ok ? CMPX_PATH_TC : -1;
  // The skinny path's counter region holds kSkinnyMaxTiles tiles; without
  // device facts (host-only path queries) assume the narrowest units.
  const int64_t sk_tiles = dev != nullptr ? skinny_tiles(g, *dev) : g.batch * ((g.N + 127) / 128);
  // (peer outputs are written by the tile kernels only)
  const bool sk_ok = ok && g.M <= 128 && sk_tiles <= kSkinnyMaxTiles && g.peers.n == 0;
  if (forced == CMPX_PATH_SKINNY) return sk_ok ? CMPX_PATH_SKINNY : -1;
  if (forced == CMPX_PATH_SIMT) return CMPX_PATH_SIMT;
  if (!ok) return CMPX_PATH_SIMT;
  // M <= 128: the single-CTA tile kernel runs one 128 x 256 tile per 256
  // columns with the whole K serial in one CTA and no split-K reduction; the
  // stream-K skinny kernel splits K over every SM.  Measured on a B200 (fp16,
  // M = 1..128, 80 shapes; single launches back to back):
  //  * T = 256-column tiles >= ~96 with K < 128 * T: the tile kernel (M 16,
  //    N 28672, K 4096: 38.9 us vs 45.2; config 4, K 8192: 5.9-6.0 TB/s vs
  //    5.85; N 32768 K 8192: 80 vs 91),
  //  * fewer tiles or deeper K: the skinny kernel (N = K = 8192: 29-41 us vs
  //    50-53; N 4096 K 14336: 26-38 vs 80-84),
  //  * 32 < M: the skinny kernel re-reads a wider A tile per unit, so the tile
  //    kernel also wins with fewer tiles (N 14336 K 4096, 56 tiles: 30 vs
  //    33-46): there the skinny kernel needs K >= 128 * T,
  //  * M < 8: the skinny kernel throughout (M 1, N 28672 K 4096: 44.6 vs 53.4).
  if (sk_ok) {
    const int64_t sms = dev != nullptr ? dev->num_sms : 148;
    const int64_t T = g.batch * ((g.N + 255) / 256);
    const bool deep = g.K >= 128 * T;
    if (g.M < 8) return CMPX_PATH_SKINNY;
    if (g.M <= 32 && (T < 96 || T >= sms || deep)) return CMPX_PATH_SKINNY;
    if (g.M > 32 && T < sms && deep) return CMPX_PATH_SKINNY;
  }
  return CMPX_PATH_TC;
}

// fp16/bf16 tile kernel choice: 0 = single-CTA 128x256 tiles, else CTA
// pairs with 256 x pair_n tiles.  Measured on a B200 (bench.py): 256x256
// pair tiles beat both alternatives on every config tried (config 3:
// 0.91 vs 0.89 single-CTA vs 0.64 for 256x128 pairs; config 2, 4096^3:
// 0.84 vs 0.77 vs 0.55), so pairs with pair_n = 256 are used whenever
// M > 128 (below that a 256-row pair tile would be at least half empty).
// CMPX_TC_PAIR=0|128|256 overrides (tuning experiments and tests).
int tc_pair_n(const Gemm& g, const DeviceInfo& dev) {
  static int forced = -2;
  if (forced == -2) {
    const char* e = std::getenv("CMPX_TC_PAIR");
    forced = -1;
    if (e != nullptr) {
      if (!std::strcmp(e, "0")) forced = 0;
      else if (!std::strcmp(e, "128")) forced = 128;
      else if (!std::strcmp(e, "256")) forced = 256;
    }
  }
  if (forced >= 0) return forced;
  return g.M <= 128 ? 0 : 256;
}

// Whether the CTA-pair kernel splits its last wave stream-K (needs the
// workspace).  Off by default: A/B on a B200 (bench.py, same session) put it
// behind whole tiles at every size tried -- 4096^3 fp16: 0.71 vs 0.82;
// bf16 2048x8192x8192: 0.72-0.79 vs 0.86; 4096x8192x8192: 0.70-0.85 vs
// 0.76-0.85 -- the partial-sum round trip through L2 costs more than the
// partial-wave tail it removes.  CMPX_TC_STREAMK=1 turns it on.
bool tc_streamk(const Gemm& g) {
  (void)g;
  static int forced = -1;
  if (forced < 0) {
    const char* e = std::getenv("CMPX_TC_STREAMK");
    forced = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return forced == 1;
}

// hi and lo splits of A and B, elem bytes each (4: tf32, 2: bf16).
size_t f32_split_bytes(const Gemm& g, size_t elem) {
  const size_t a = size_t(g.batch) * size_t(g.M) * size_t(g.K);
  const size_t b = size_t(g.batch) * size_t(g.K) * size_t(g.N);
  auto up = [elem](size_t x) { return (x * elem + 255) / 256 * 256; };
  return 2 * up(a) + 2 * up(b);
}

size_t workspace_for(const Gemm& g, int path, const DeviceInfo& dev) {
  if (path == CMPX_PATH_SKINNY) return skinny_workspace_bytes(g, dev);
  if (path == CMPX_PATH_TC && g.dtype == CMPX_F32) return f32_split_bytes(g, 4);
  if (path == CMPX_PATH_BF16X3) return f32_split_bytes(g, 2);
  if (path == CMPX_PATH_TC) {
    const int pair_n = tc_pair_n(g, dev);
    return (pair_n > 0 && tc_streamk(g)) ? tc2_workspace_bytes(g, pair_n, dev) : 0;
  }
  return 0;
}

int run_gemm(const cmpx_gemm_args* args, cudaStream_t s) {
  int st = validate(args);
  if (st != CMPX_OK) return st;
  if (args->batch == 0 || args->M == 0 || args->N == 0) return CMPX_OK;
  DeviceState* d = nullptr;
  st = device_state(&d);
  if (st != CMPX_OK) return st;
  const Gemm g = to_gemm(args);
  const int path = choose_path(g, args->path, &d->info);
  if (path < 0) return CMPX_ERR_UNSUPPORTED;
  // The multicast output is written by the CTA-pair kernel's epilogue only.
  if (g.mc_C != nullptr && (g.dtype == CMPX_F32 || path != CMPX_PATH_TC || g.K == 0 ||
                            tc_pair_n(g, d->info) == 0 || g.N % 8 != 0 || (g.ldc * 2) % 16 != 0 ||
                            (reinterpret_cast<uintptr_t>(g.mc_C) & 15u) != 0))
    return CMPX_ERR_UNSUPPORTED;
  if (g.K == 0) return cuda_status(launch_fill_bias(g, s));
  if (path == CMPX_PATH_SIMT) return cuda_status(launch_simt(g, s));

  void* ws = nullptr;
  const size_t need = workspace_for(g, path, d->info);
  if (need > 0) {
    if (args->workspace != nullptr) {
      if (args->workspace_bytes < need) return CMPX_ERR_WORKSPACE;
      if (!aligned16(args->workspace)) return CMPX_ERR_INVALID_ARG;
      ws = args->workspace;
    } else {
      // slot 1 keeps its counter region zero between calls (skinny and
      // CTA-pair stream-K); slot 0 is plain scratch (3xTF32 splits)
      st = library_workspace(*d, g.dtype == CMPX_F32 ? 0 : 1, need, &ws);
      if (st != CMPX_OK) return st;
    }
  }

  if (path == CMPX_PATH_SKINNY) {
    const uint32_t mn = uint32_t(skinny_mn(g.M));
    CUtensorMap tB, tA;
    st = g.b_kmajor ? encode_3d(&tB, g.dtype, g.B, g.K, g.N, g.batch, g.ldb, g.sb, 64, 128)
                    : encode_3d(&tB, g.dtype, g.B, g.N, g.K, g.batch, g.ldb, g.sb, 64, 128);
    if (st != CMPX_OK) return st;
    st = encode_3d(&tA, g.dtype, g.A, g.K, g.M, g.a_bcast ? 1 : g.batch, g.lda, g.sa, 64, mn);
    if (st != CMPX_OK) return st;
    return cuda_status(launch_skinny(g, tB, tA, ws, d->info, d->err_word, s));
  }

  if (g.dtype != CMPX_F32) {
    CUtensorMap tA, tB;
    st = encode_3d(&tA, g.dtype, g.A, g.K, g.M, g.a_bcast ? 1 : g.batch, g.lda, g.sa, 64, 128);
    if (st != CMPX_OK) return st;
    const int pair_n = tc_pair_n(g, d->info);
    if (pair_n > 0) {
      st = g.b_kmajor ? encode_3d(&tB, g.dtype, g.B, g.K, g.N, g.batch, g.ldb, g.sb, 64, uint32_t(pair_n / 2))
                      : encode_3d(&tB, g.dtype, g.B, g.N, g.K, g.batch, g.ldb, g.sb, 64, 64);
      if (st != CMPX_OK) return st;
      if (g.peers.n > 0) {
        // Output also goes to peer GPUs: staged TMA stores (bulk NVLink writes).
        OutMaps om{};
        om.n = 1 + g.peers.n;
        if ((st = encode_out_map(&om.m[0], g, g.C)) != CMPX_OK) return st;
        for (int i = 0; i < g.peers.n; ++i)
          if ((st = encode_out_map(&om.m[1 + i], g, g.peers.base[i])) != CMPX_OK) return st;
        return cuda_status(launch_tc2_f16(g, tA, tB, pair_n, ws, d->info, d->err_word, s, &om));
      }
      return cuda_status(launch_tc2_f16(g, tA, tB, pair_n, ws, d->info, d->err_word, s));
    }
    st = g.b_kmajor ? encode_3d(&tB, g.dtype, g.B, g.K, g.N, g.batch, g.ldb, g.sb, 64, 256)
                    : encode_3d(&tB, g.dtype, g.B, g.N, g.K, g.batch, g.ldb, g.sb, 64, 64);
    if (st != CMPX_OK) return st;
    return cuda_status(launch_tc_f16(g, tA, tB, 256, d->info, d->err_word, s));
  }

  // fp32: split A and B into packed hi/lo operands (tf32 for 3xTF32, bf16
  // for bf16x3), then three products per k on the tensor cores.  B is always
  // stored K-major ([N][K]) by the pre-pass: a [K,N] source is transposed
  // while it is split.
  const bool bf = path == CMPX_PATH_BF16X3;
  const size_t elem = bf ? 2 : 4;
  const size_t a_elems = size_t(g.batch) * size_t(g.M) * size_t(g.K);
  const size_t b_elems = size_t(g.batch) * size_t(g.K) * size_t(g.N);
  auto up = [elem](size_t x) { return (x * elem + 255) / 256 * 256; };
  uint8_t* base = reinterpret_cast<uint8_t*>(ws);
  void* a_hi = base;
  void* a_lo = base + up(a_elems);
  void* b_hi = base + 2 * up(a_elems);
  void* b_lo = base + 2 * up(a_elems) + up(b_elems);
  const int64_t a_batch = g.a_bcast ? 1 : g.batch;  // a shared A is split once
  const int64_t b_rows = g.b_kmajor ? g.N : g.K, b_cols = g.b_kmajor ? g.K : g.N;
  const float* fA = reinterpret_cast<const float*>(g.A);
  const float* fB = reinterpret_cast<const float*>(g.B);
  cudaError_t e;
  // bf16x3 keeps the splits of a [K,N] B N-major (no transpose) when packed
  // rows of N are 16-byte multiples and the source suits the vector split.
  const bool b_nmajor = bf && !g.b_kmajor && g.N % 8 == 0 && g.ldb % 4 == 0 && aligned16(g.B) &&
                        (g.batch <= 1 || g.sb % 4 == 0);
  if (bf) {
    e = launch_split_bf16(fA, a_hi, a_lo, a_batch, g.M, g.K, g.lda, g.sa, false, d->info.num_sms, s);
    if (e == cudaSuccess)
      e = launch_split_bf16(fB, b_hi, b_lo, g.batch, b_rows, b_cols, g.ldb, g.sb, !g.b_kmajor && !b_nmajor,
                            d->info.num_sms, s);
  } else {
    e = launch_split_tf32(fA, static_cast<float*>(a_hi), static_cast<float*>(a_lo), a_batch, g.M, g.K, g.lda, g.sa,
                          false, d->info.num_sms, s);
    if (e == cudaSuccess)
      e = launch_split_tf32(fB, static_cast<float*>(b_hi), static_cast<float*>(b_lo), g.batch, b_rows, b_cols, g.ldb,
                            g.sb, !g.b_kmajor, d->info.num_sms, s);
  }
  if (e != cudaSuccess) return CMPX_ERR_CUDA;
  CUtensorMap tA, tA2, tB, tB2;
  const uint64_t sa = uint64_t(g.M) * uint64_t(g.K), sb = uint64_t(g.N) * uint64_t(g.K);
  const int op = bf ? CMPX_BF16 : CMPX_F32;     // element type of the packed operands
  const uint32_t box_k = bf ? 64 : 32;          // one 128-byte swizzle row of K
  if ((st = encode_3d(&tA, op, a_hi, g.K, g.M, a_batch, g.K, sa, box_k, 128)) != CMPX_OK) return st;
  if ((st = encode_3d(&tA2, op, a_lo, g.K, g.M, a_batch, g.K, sa, box_k, 128)) != CMPX_OK) return st;
  if (b_nmajor) {  // [K][N] splits: 64-column x 64-row boxes, N-major chunks
    if ((st = encode_3d(&tB, op, b_hi, g.N, g.K, g.batch, g.N, sb, 64, 64)) != CMPX_OK) return st;
    if ((st = encode_3d(&tB2, op, b_lo, g.N, g.K, g.batch, g.N, sb, 64, 64)) != CMPX_OK) return st;
  } else {
    const uint32_t box_n = bf ? 128u : uint32_t(tf32x3_block_n());  // rows of B per tile
    if ((st = encode_3d(&tB, op, b_hi, g.K, g.N, g.batch, g.K, sb, box_k, box_n)) != CMPX_OK) return st;
    if ((st = encode_3d(&tB2, op, b_lo, g.K, g.N, g.batch, g.K, sb, box_k, box_n)) != CMPX_OK) return st;
  }
  if (bf) return cuda_status(launch_tc_bf16x3(g, tA, tA2, tB, tB2, b_nmajor, d->info, d->err_word, s));
  return cuda_status(launch_tc_tf32x3(g, tA, tA2, tB, tB2, d->info, d->err_word, s));
}

int packed_matmul(int dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                  cudaStream_t s) {
  cmpx_gemm_args a;
  std::memset(&a, 0, sizeof(a));
  a.dtype = dtype;
  a.A = A;
  a.B = B;
  a.C = C;
  a.batch = 1;
  a.M = M;
  a.N = N;
  a.K = K;
  a.lda = K;
  a.ldb = N;
  a.ldc = N;
  a.b_layout = CMPX_B_KN;
  return run_gemm(&a, s);
}

}  // namespace

// The CTA-pair GEMM with column-progress flags (gather_ce.cu): fp16/bf16,
// one 256-column pair-tile kernel launch, whole tiles only (every tile
// counts into its flag), no peer stores.
int run_gemm_flagged(const cmpx_gemm_args* args, int* flags, int flag_tiles, cudaStream_t s) {
  int st = validate(args);
  if (st != CMPX_OK) return st;
  if (args->batch == 0 || args->M == 0 || args->N == 0) return CMPX_OK;
  DeviceState* d = nullptr;
  st = device_state(&d);
  if (st != CMPX_OK) return st;
  Gemm g = to_gemm(args);
  g.col_flags = flags;
  g.flag_tiles = flag_tiles;
  if (g.dtype == CMPX_F32 || choose_path(g, args->path, &d->info) != CMPX_PATH_TC) return CMPX_ERR_UNSUPPORTED;
  if (tc_pair_n(g, d->info) != 256) return CMPX_ERR_UNSUPPORTED;
  CUtensorMap tA, tB;
  st = encode_3d(&tA, g.dtype, g.A, g.K, g.M, g.a_bcast ? 1 : g.batch, g.lda, g.sa, 64, 128);
  if (st != CMPX_OK) return st;
  st = g.b_kmajor ? encode_3d(&tB, g.dtype, g.B, g.K, g.N, g.batch, g.ldb, g.sb, 64, 128)
                  : encode_3d(&tB, g.dtype, g.B, g.N, g.K, g.batch, g.ldb, g.sb, 64, 64);
  if (st != CMPX_OK) return st;
  return cuda_status(launch_tc2_f16(g, tA, tB, 256, nullptr, d->info, d->err_word, s));
}

// CMPX_PDL=0 turns programmatic dependent launch off (A/B measurements).
bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("CMPX_PDL");
    on = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

unsigned epilogue_sleep_ns() {
  static long v = -1;
  if (v < 0) {
    const char* e = std::getenv("CMPX_EPI_SLEEP_NS");
    long x = e != nullptr ? std::strtol(e, nullptr, 10) : 0;
    v = x < 0 ? 0 : (x > 100000 ? 100000 : x);
  }
  return unsigned(v);
}

int tf32x3_block_n() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("CMPX_TF32_BN");
    v = (e != nullptr && std::strcmp(e, "128") == 0) ? 128 : 256;
  }
  return v;
}

int tc2_group_m() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("CMPX_TC_GROUP_M");
    const long x = e != nullptr ? std::strtol(e, nullptr, 10) : 8;
    v = x < 1 ? 1 : (x > 64 ? 64 : int(x));
  }
  return v;
}

int* device_error_word() {
  DeviceState* d = nullptr;
  return device_state(&d) == CMPX_OK ? d->err_word : nullptr;
}

int device_facts(DeviceInfo* info, int** err_word) {
  DeviceState* d = nullptr;
  const int st = device_state(&d);
  if (st != CMPX_OK) return st;
  *info = d->info;
  *err_word = d->err_word;
  return CMPX_OK;
}

int encode_tmap_3d(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t rows, uint64_t batch,
                   uint64_t ld, uint64_t bstride, uint32_t box_inner, uint32_t box_rows) {
  return encode_3d(m, dtype, base, inner, rows, batch, ld, bstride, box_inner, box_rows);
}

}  // namespace cmpx

using namespace cmpx;

extern "C" {

int cmpx_matmul_f16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, cmpx_stream_t stream) {
  return packed_matmul(CMPX_F16, A, B, C, M, N, K, stream);
}

int cmpx_matmul_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, cmpx_stream_t stream) {
  return packed_matmul(CMPX_BF16, A, B, C, M, N, K, stream);
}

int cmpx_matmul_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                    cmpx_stream_t stream) {
  return packed_matmul(CMPX_F32, A, B, C, M, N, K, stream);
}

int cmpx_gemm(const cmpx_gemm_args* args, cmpx_stream_t stream) {
  // Kernels index the batch with a grid dimension (at most 65535); larger
  // batches run as consecutive slices of it.
  constexpr int64_t kMaxBatch = 65535;
  if (args == nullptr || args->batch <= kMaxBatch) return run_gemm(args, stream);
  const int st = validate(args);
  if (st != CMPX_OK) return st;
  const int64_t E = args->dtype == CMPX_F32 ? 4 : 2;
  for (int64_t b0 = 0; b0 < args->batch; b0 += kMaxBatch) {
    cmpx_gemm_args part = *args;
    part.batch = std::min<int64_t>(kMaxBatch, args->batch - b0);
    part.A = static_cast<const char*>(args->A) + b0 * args->stride_a * E;
    part.B = static_cast<const char*>(args->B) + b0 * args->stride_b * E;
    part.C = static_cast<char*>(args->C) + b0 * args->stride_c * E;
    const int r = run_gemm(&part, stream);
    if (r != CMPX_OK) return r;
  }
  return CMPX_OK;
}

size_t cmpx_gemm_workspace_size(const cmpx_gemm_args* args) {
  if (validate(args) != CMPX_OK) return 0;
  if (args->batch == 0 || args->M == 0 || args->N == 0) return 0;
  DeviceState* d = nullptr;
  if (device_state(&d) != CMPX_OK) return 0;
  const Gemm g = to_gemm(args);
  const int path = choose_path(g, args->path, &d->info);
  if (path < 0) return 0;
  return workspace_for(g, path, d->info);
}

int cmpx_gemm_select_path(const cmpx_gemm_args* args) {
  if (validate(args) != CMPX_OK) return -1;
  const Gemm g = to_gemm(args);
  return choose_path(g, args->path, nullptr);
}

int cmpx_add_bias(int dtype, void* C, const void* bias, int64_t rows, int64_t cols, cmpx_stream_t stream) {
  if (dtype != CMPX_F16 && dtype != CMPX_BF16 && dtype != CMPX_F32) return CMPX_ERR_INVALID_ARG;
  if (rows < 0 || cols < 0) return CMPX_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return CMPX_OK;
  if (C == nullptr || bias == nullptr) return CMPX_ERR_INVALID_ARG;
  return cuda_status(launch_add_bias(dtype, C, bias, rows, cols, stream));
}

int cmpx_device_error(int* code) {
  if (code == nullptr) return CMPX_ERR_INVALID_ARG;
  *code = 0;
  int* w = device_error_word();
  if (w == nullptr) return CMPX_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return CMPX_ERR_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return CMPX_ERR_CUDA;
  if (v != 0) {
    const int zero = 0;
    if (cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return CMPX_ERR_CUDA;
    // A launch that gave up may have left split-K counters or the piece
    // claim counter non-zero: restore the library workspace's counter region
    // (caller workspaces are the caller's to re-zero).
    DeviceState* d = nullptr;
    if (device_state(&d) == CMPX_OK) {
      std::lock_guard<std::mutex> lk(d->ws_mu);
      for (int slot = 0; slot < 2; ++slot)
        if (d->ws[slot] != nullptr && d->ws_bytes[slot] >= kSkinnyCounterBytes &&
            cudaMemset(d->ws[slot], 0, kSkinnyCounterBytes) != cudaSuccess)
          return CMPX_ERR_CUDA;
    }
  }
  *code = v;
  return CMPX_OK;
}

const char* cmpx_status_string(int status) {
  switch (status) {
    case CMPX_OK: return "ok";
    case CMPX_ERR_INVALID_ARG: return "invalid argument";
    case CMPX_ERR_UNSUPPORTED: return "unsupported shape, alignment, path or device";
    case CMPX_ERR_CUDA: return "CUDA error";
    case CMPX_ERR_NO_MEMORY: return "out of device memory for workspace";
    case CMPX_ERR_DEVICE: return "device-side error (bounded wait expired)";
    case CMPX_ERR_WORKSPACE: return "workspace too small";
    case CMPX_ERR_TOO_LARGE: return "problem larger than the fixed scratch of cmpx_matmul_skinny_noalloc";
    default: return "unknown status";
  }
}

const char* cmpx_version(void) { return "cmpx 0.1.0 sm_100a"; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Reference-compatible C++-linkage launchers (same signatures as
// src/main.cpp:12-19).  Legacy default stream, no return value; a failure is
// reported on stderr, as the reference's fp32 launcher does
// (src/cuda/fp32_matmul.cu:260-264).
static void report(const char* what, int st) {
  if (st != CMPX_OK) std::fprintf(stderr, "cmpx %s error: %s\n", what, cmpx_status_string(st));
}

CMPX_API void launch_matmul_fp16(const void* input, const void* weight, void* output, int M, int N, int K) {
  report("launch_matmul_fp16", cmpx_matmul_f16(input, weight, output, M, N, K, nullptr));
}
CMPX_API void launch_matmul_fp32(const float* input, const float* weight, float* output, int M, int N, int K) {
  report("launch_matmul_fp32", cmpx_matmul_f32(input, weight, output, M, N, K, nullptr));
}
CMPX_API void launch_matmul_bf16(const void* input, const void* weight, void* output, int M, int N, int K) {
  report("launch_matmul_bf16", cmpx_matmul_bf16(input, weight, output, M, N, K, nullptr));
}
CMPX_API void launch_add_bias_fp16(void* output, const void* bias, int rows, int cols) {
  report("launch_add_bias_fp16", cmpx_add_bias(CMPX_F16, output, bias, rows, cols, nullptr));
}
CMPX_API void launch_add_bias_fp32(float* output, const float* bias, int rows, int cols) {
  report("launch_add_bias_fp32", cmpx_add_bias(CMPX_F32, output, bias, rows, cols, nullptr));
}
CMPX_API void launch_add_bias_bf16(void* output, const void* bias, int rows, int cols) {
  report("launch_add_bias_bf16", cmpx_add_bias(CMPX_BF16, output, bias, rows, cols, nullptr));
}
