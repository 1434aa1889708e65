// Swap-AB, stream-K tcgen05 GEMM for skinny M (decode shapes, M <= 128).
//
// The reference runs every shape through its 128x128 SIMT tile kernel
// (src/cuda/fp16_matmul.cu:63-283, bf16: src/cuda/bf16_matmul.cu:51-226);
// at M = 16 127/128 of each tile is zero padding and the B operand (the
// weight, hundreds of MB) is streamed by only N/128 CTAs.  Here the product is
// computed transposed, C^T[N, M] = B^T[N, K] * A^T[K, M]:
//   * the 128-row MMA operand is a 128-column slab of B (N fills MMA-M),
//   * the narrow MMA operand is A (MMA-N = M rounded up to 16/32/64),
// and the (N-tile, k-block) work units are split evenly over one CTA per SM
// (stream-K), so every SM streams an equal share of B from HBM.  A tile whose
// k-range is split between CTAs is reduced deterministically: each part
// writes fp32 partials to a workspace slot, and the last part to arrive
// (per-tile counter) sums the parts in CTA order, adds the bias, rounds once
// and stores.  The counters are left at zero for the next launch.
//
// Shared-memory operand layouts (128-byte swizzle, written by TMA):
//   B slab, [K,N] source: 2 chunks of [128 K rows][64 N] (MN-major, LBO 16384, SBO 1024)
//   B slab, [N,K] source: 2 atoms of [128 N rows][64 K]   (K-major, SBO 1024, atoms 16 KB apart)
//   A tile            : 2 atoms of [MN rows][64 K]        (K-major, SBO 1024, atoms MN*128 B apart)
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace cmpx {
namespace {

struct SkParams {
  void* C;
  const void* bias;
  int M, N, K, batch;
  long long ldc, stride_c;
  int n_tiles;    // N-tiles per batch entry
  int kbt;        // k-blocks per tile
  long long units;  // batch * n_tiles * kbt
  float* ws;      // [grid][2 slots][NS][MN/4][128 n][4] fp32 partials
  int* counters;  // [batch * n_tiles][4] (one per epilogue warp quadrant)
  int a_bcast;
  int bias_m;
  int* err;
};

// NS = number of 128-column sub-slabs per work unit (tile width 128*NS).
// Each pipeline stage holds one sub-slab (and a copy of the A tile), so the
// stage size -- and with it the pipeline depth -- does not depend on NS,
// while a CTA's consecutive stages walk NS*256 contiguous bytes of each B row
// ([K,N] layout) before moving down to the next k-block.
template <int FMT, bool B_KMAJOR, int MN, int NS>
struct SkCfg {
  // 128 K rows per k-block: in this kernel's walk down a column strip of B,
  // TMA boxes of 128 rows stream from HBM at ~6.5 TB/s where 64-row boxes
  // reach only ~3.5 (measured on a B200 with a no-compute TMA stream).
  static constexpr int BK = 128;
  static constexpr int SUB_BYTES = 128 * 256;       // 128 N x 128 K x 2 B (two 16 KB boxes / atoms)
  static constexpr int ATILE_BYTES = MN * 256;      // MN rows x 128 K x 2 B (two 64-K atoms)
  static constexpr int STAGE_BYTES = SUB_BYTES + ATILE_BYTES;
  static constexpr int STAGES_FIT = (225 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 16 ? 16 : STAGES_FIT;
  static constexpr int ACC_COLS = NS * MN;          // one accumulator buffer
  static constexpr uint32_t TMEM_COLS = (2 * ACC_COLS) < 32 ? 32 : 2 * ACC_COLS;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t IDESC = make_idesc(uint32_t(FMT), B_KMAJOR ? 0u : 1u, 0u, 128, MN);
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
  static_assert(STAGES >= 2, "pipeline depth");
  static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
};

__device__ __forceinline__ long long unit_begin(long long g, long long U, long long G) { return g * U / G; }
// CTA owning unit u: the largest g with unit_begin(g) <= u.
__device__ __forceinline__ long long unit_owner(long long u, long long U, long long G) {
  return ((u + 1) * G - 1) / U;
}

__device__ __forceinline__ void record_error(int* err, volatile int* abort, int code) {
  *abort = 1;
  atomicCAS(err, 0, code);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ void from_f32(float v, __half* o) { *o = __float2half_rn(v); }
__device__ __forceinline__ void from_f32(float v, __nv_bfloat16* o) { *o = __float2bfloat16_rn(v); }

template <int FMT, bool B_KMAJOR, int MN, int NS>
__global__ void __launch_bounds__(192, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                       const SkParams p) {
  using Cfg = SkCfg<FMT, B_KMAJOR, MN, NS>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int EC = MN < 32 ? MN : 32;  // epilogue column chunk
  using T = typename std::conditional<FMT == 0, __half, __nv_bfloat16>::type;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + size_t(STAGES) * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_trigger();
  pdl_wait();

  const long long G = gridDim.x;
  const long long U = p.units;
  const long long u_begin = unit_begin(blockIdx.x, U, G);
  const long long u_end = unit_begin(blockIdx.x + 1, U, G);
  const int kbt = p.kbt;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmB);
      prefetch_tmap(&tmA);
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (long long u = u_begin; u < u_end && ok; ++u) {
        const long long tile = u / kbt;
        const int kb = int(u - tile * kbt);
        const int b = int(tile / p.n_tiles);
        const int n0 = int(tile - 1LL * b * p.n_tiles) * (128 * NS);
        const int k0 = kb * Cfg::BK;
        for (int sub = 0; sub < NS && ok; ++sub) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            record_error(p.err, abort_flag, kDevTimeoutEmpty);
            ok = false;
            break;
          }
          uint8_t* sB = smem + size_t(stage) * Cfg::STAGE_BYTES;
          uint8_t* sA = sB + Cfg::SUB_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (B_KMAJOR)  // [N,K]: box = 64 K x 128 rows -> K-major atom h (K 64h..64h+63)
              tma_load_3d(sB + h * 16384, &tmB, &full_bar[stage], k0 + 64 * h, n0 + sub * 128, b);
            else  // [K,N]: box = 64 N x 128 K rows -> MN-major chunk h (N 64h..64h+63)
              tma_load_3d(sB + h * 16384, &tmB, &full_bar[stage], n0 + sub * 128 + 64 * h, k0, b);
            tma_load_3d(sA + h * (MN * 128), &tmA, &full_bar[stage], k0 + 64 * h, 0, p.a_bcast ? 0 : b);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        const uint32_t n = issued < uint32_t(STAGES) ? issued : uint32_t(STAGES);
        uint32_t s = stage, ph = phase;
        volatile int never = 0;
        for (uint32_t i = 0; i < n; ++i) {
          if (s == 0) {
            s = STAGES - 1;
            ph ^= 1;
          } else {
            --s;
          }
          mbar_wait(&full_bar[s], ph, &never);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int ls = 0;  // local segment counter
      for (long long u = u_begin; u < u_end && ok; ++ls) {
        const long long tile = u / kbt;
        const int kb0 = int(u - tile * kbt);
        const int kb1 = int(min((long long)kbt, (long long)kb0 + (u_end - u)));
        u += kb1 - kb0;
        const int acc = ls & 1;
        const uint32_t acc_phase = (ls >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag)) {
          record_error(p.err, abort_flag, kDevTimeoutAccEmpty);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * Cfg::ACC_COLS);
        for (int kb = kb0; kb < kb1 && ok; ++kb) {
          for (int sub = 0; sub < NS; ++sub) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
              record_error(p.err, abort_flag, kDevTimeoutFull);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b_addr = smem_u32(smem + size_t(stage) * Cfg::STAGE_BYTES);
            const uint32_t a_addr = b_addr + Cfg::SUB_BYTES;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              // 16 K per MMA: K-major operands step 32 B inside a 64-K atom,
              // then move to the next atom; the MN-major slab steps 16 rows.
              const uint64_t a_desc = make_sdesc_sw128(a_addr + (ks >> 2) * (MN * 128) + (ks & 3) * 32, 16, 1024);
              const uint64_t slab_desc =
                  B_KMAJOR ? make_sdesc_sw128(b_addr + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024)
                           : make_sdesc_sw128(b_addr + ks * 2048, 16384, 1024);
              mma_f16(d_tmem + sub * MN, slab_desc, a_desc, Cfg::IDESC, (kb != kb0 || ks != 0) ? 1u : 0u);
            }
            mma_commit(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        if (ok) mma_commit(&acc_full[acc]);
      }
      if (!ok) {
        mma_commit(drain_bar);
        volatile int never = 0;
        mbar_wait(drain_bar, 0, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int et = q * 32 + lane;  // TMEM lane this thread reads == n offset in the slab
    T* C = reinterpret_cast<T*>(p.C);
    const T* bias = reinterpret_cast<const T*>(p.bias);
    const long long first_tile = u_begin / kbt;
    int ls = 0;
    for (long long u = u_begin; u < u_end; ++ls) {
      const long long tile = u / kbt;
      const int kb0 = int(u - tile * kbt);
      const int kb1 = int(min((long long)kbt, (long long)kb0 + (u_end - u)));
      u += kb1 - kb0;
      const int b = int(tile / p.n_tiles);
      const int nt0 = int(tile - 1LL * b * p.n_tiles) * (128 * NS) + et;  // n of sub-slab 0
      const int acc = ls & 1;
      const uint32_t acc_phase = (ls >> 1) & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, abort_flag));
      if (!ok) {
        if (lane == 0) record_error(p.err, abort_flag, kDevTimeoutAccFull);
        break;
      }
      tc_fence_after();
      const long long t_u0 = tile * kbt;
      const long long g_lo = unit_owner(t_u0, U, G);
      const long long g_hi = unit_owner(t_u0 + kbt - 1, U, G);
      const bool whole = g_lo == g_hi;  // whole k-range of the tile in this CTA
      const int slot = (tile == first_tile) ? 0 : 1;
      T* cb = C + size_t(b) * p.stride_c;
      const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * Cfg::ACC_COLS);
#pragma unroll 1
      for (int sub = 0; sub < NS; ++sub) {
        // Columns (rows of C) in chunks of EC so no MN-float array stays live.
        const int n = nt0 + sub * 128;
        float* part = p.ws + (((size_t(blockIdx.x) * 2 + slot) * NS + sub) * MN) * 128;
        const float bv = (whole && n < p.N && bias != nullptr && !p.bias_m) ? to_f32<T>(bias[n]) : 0.0f;
#pragma unroll 1
        for (int c0 = 0; c0 < MN; c0 += EC) {
          float v[EC];
#pragma unroll
          for (int c = 0; c < EC; c += 16) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(t_row + sub * MN + c0 + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[c + i] = __uint_as_float(r[i]);
          }
          if (whole) {
            // column n of C^T is C[:, n]: lanes write consecutive n (coalesced)
            if (n < p.N) {
#pragma unroll
              for (int j = 0; j < EC; ++j)
                if (c0 + j < p.M) {
                  const float rb = (bias != nullptr && p.bias_m) ? to_f32<T>(bias[c0 + j]) : 0.0f;
                  from_f32(v[j] + bv + rb, cb + size_t(c0 + j) * p.ldc + n);
                }
            }
          } else {
            // [MN/4][128 n][4] partials: a float4 per lane, 512 contiguous
            // bytes per warp store
            float4* dst = reinterpret_cast<float4*>(part) + size_t(c0 / 4) * 128 + et;
#pragma unroll
            for (int j = 0; j < EC; j += 4)
              __stcg(dst + (j / 4) * 128, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);  // TMEM buffer free for the segment after next

      if (!whole) {
        // Each epilogue warp owns 32 lanes (n values) of every sub-slab and
        // reduces them independently: per-(tile, quadrant) counters, no CTA
        // barrier.  The last of the tile's parts to arrive sums all parts in
        // CTA order (deterministic), adds the bias, rounds once and stores.
        __threadfence();
        __syncwarp();
        int prev = 0;
        if (lane == 0) prev = atomicAdd(p.counters + tile * 4 + q, 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == int(g_hi - g_lo)) {
          __threadfence();
          // Only the first owner's range can start before this tile (its
          // part then sits in that CTA's second slot); later owners start
          // inside the tile and use their first slot.
          const int sl_lo = unit_begin(g_lo, U, G) < tile * kbt ? 1 : 0;
          const size_t slot_floats = size_t(NS) * MN * 128;
#pragma unroll 1
          for (int sub = 0; sub < NS; ++sub) {
            const int n = nt0 + sub * 128;
            const float bv = (n < p.N && bias != nullptr && !p.bias_m) ? to_f32<T>(bias[n]) : 0.0f;
#pragma unroll 1
            for (int c0 = 0; c0 < MN; c0 += EC) {
              float acc_s[EC];
#pragma unroll
              for (int j = 0; j < EC; ++j) acc_s[j] = 0.0f;
              const size_t lane_off = size_t(sub) * MN * 128 + (size_t(c0 / 4) * 128 + et) * 4;
              // parts summed in CTA order; unrolled so several parts' loads
              // are in flight at once
#pragma unroll 4
              for (long long gg = g_lo; gg <= g_hi; ++gg) {
                const int sl = gg == g_lo ? sl_lo : 0;
                const float4* pp =
                    reinterpret_cast<const float4*>(p.ws + (size_t(gg) * 2 + sl) * slot_floats + lane_off);
#pragma unroll
                for (int j = 0; j < EC; j += 4) {
                  const float4 x = __ldcg(pp + (j / 4) * 128);
                  acc_s[j] += x.x;
                  acc_s[j + 1] += x.y;
                  acc_s[j + 2] += x.z;
                  acc_s[j + 3] += x.w;
                }
              }
              if (n < p.N) {
#pragma unroll
                for (int j = 0; j < EC; ++j)
                  if (c0 + j < p.M) {
                    const float rb = (bias != nullptr && p.bias_m) ? to_f32<T>(bias[c0 + j]) : 0.0f;
                    from_f32(acc_s[j] + bv + rb, cb + size_t(c0 + j) * p.ldc + n);
                  }
              }
            }
          }
          if (lane == 0) p.counters[tile * 4 + q] = 0;
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int FMT, bool B_KMAJOR, int MN, int NS>
cudaError_t launch_sk_impl(const Gemm& g, const CUtensorMap& tB, const CUtensorMap& tA, void* ws,
                           const DeviceInfo& dev, int* dev_err, cudaStream_t s) {
  using Cfg = SkCfg<FMT, B_KMAJOR, MN, NS>;
  auto kern = gemm_skinny_kernel<FMT, B_KMAJOR, MN, NS>;
  static_assert(Cfg::SMEM <= 232448, "shared memory budget");
  static unsigned long long smem_set = 0;  // one flag word per kernel instantiation
  cudaError_t e = set_smem_once(kern, int(Cfg::SMEM), smem_set);
  if (e != cudaSuccess) return e;
  SkParams p;
  p.C = g.C;
  p.bias = g.bias;
  p.M = int(g.M);
  p.N = int(g.N);
  p.K = int(g.K);
  p.batch = int(g.batch);
  p.ldc = g.ldc;
  p.stride_c = g.sc;
  p.n_tiles = int((g.N + 128 * NS - 1) / (128 * NS));
  p.kbt = int((g.K + Cfg::BK - 1) / Cfg::BK);
  p.units = 1LL * g.batch * p.n_tiles * p.kbt;
  const long long grid = p.units < dev.num_sms ? p.units : dev.num_sms;
  p.counters = reinterpret_cast<int*>(ws);
  p.ws = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kSkinnyCounterBytes);
  p.a_bcast = g.a_bcast;
  p.bias_m = g.bias_m;
  p.err = dev_err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  apply_pdl(cfg, attr, 0);
  return cudaLaunchKernelEx(&cfg, kern, tB, tA, p);
}

template <int FMT, bool B_KMAJOR, int MN>
cudaError_t launch_sk_ns(const Gemm& g, const CUtensorMap& tB, const CUtensorMap& tA, void* ws,
                         const DeviceInfo& dev, int* dev_err, cudaStream_t s) {
  switch (skinny_ns(g, dev)) {
    case 8:
      if constexpr (MN <= 32) return launch_sk_impl<FMT, B_KMAJOR, MN, 8>(g, tB, tA, ws, dev, dev_err, s);
      return cudaErrorInvalidValue;
    case 4:
      if constexpr (MN <= 64) return launch_sk_impl<FMT, B_KMAJOR, MN, 4>(g, tB, tA, ws, dev, dev_err, s);
      return cudaErrorInvalidValue;
    case 2: return launch_sk_impl<FMT, B_KMAJOR, MN, 2>(g, tB, tA, ws, dev, dev_err, s);
    default: return launch_sk_impl<FMT, B_KMAJOR, MN, 1>(g, tB, tA, ws, dev, dev_err, s);
  }
}

template <int FMT, bool B_KMAJOR>
cudaError_t launch_sk_mn(const Gemm& g, const CUtensorMap& tB, const CUtensorMap& tA, void* ws,
                         const DeviceInfo& dev, int* dev_err, cudaStream_t s) {
  switch (skinny_mn(g.M)) {
    case 16: return launch_sk_ns<FMT, B_KMAJOR, 16>(g, tB, tA, ws, dev, dev_err, s);
    case 32: return launch_sk_ns<FMT, B_KMAJOR, 32>(g, tB, tA, ws, dev, dev_err, s);
    case 64: return launch_sk_ns<FMT, B_KMAJOR, 64>(g, tB, tA, ws, dev, dev_err, s);
    default: return launch_sk_ns<FMT, B_KMAJOR, 128>(g, tB, tA, ws, dev, dev_err, s);
  }
}

}  // namespace

int skinny_mn(int64_t M) { return M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128)); }

// Sub-slabs per work unit.  Measured on config 4 (16 x 28672 x 8192 fp16,
// B200, 128-row k-blocks): 1 sub-slab 5221 GB/s single launch / 5657
// back-to-back, 2 -> 5082 / 5452, 4 -> 4596 / 4933, so one 128-column slab
// per unit is used.  CMPX_SKINNY_NS=1|2|4|8 overrides (tuning experiments;
// NS * M rounded up must fit 256 TMEM columns).
int skinny_ns(const Gemm& g, const DeviceInfo& dev) {
  (void)dev;
  const int mn = skinny_mn(g.M);
  static int forced = -1;
  if (forced < 0) {
    const char* e = std::getenv("CMPX_SKINNY_NS");
    forced = 0;
    if (e != nullptr && (e[0] == '1' || e[0] == '2' || e[0] == '4' || e[0] == '8') && e[1] == 0) forced = e[0] - '0';
  }
  if (forced > 0 && forced * mn <= 256) return forced;
  return 1;
}

size_t skinny_partials_bytes(const DeviceInfo& dev, int ns, int mn) {
  return size_t(dev.num_sms) * 2 * size_t(ns) * size_t(mn) * 128 * 4;
}

int64_t skinny_tiles(const Gemm& g, const DeviceInfo& dev) {
  const int ns = skinny_ns(g, dev);
  return g.batch * ((g.N + 128 * ns - 1) / (128 * ns));
}

// A fixed-size counter region (one int per tile and epilogue warp, for up to
// kSkinnyMaxTiles tiles) at offset 0, then the fp32 partials.  Every call
// leaves the counters it used at zero; keeping the region at a fixed place
// means partials of one call never land on counters of another.
size_t skinny_workspace_bytes(const Gemm& g, const DeviceInfo& dev) {
  return kSkinnyCounterBytes + skinny_partials_bytes(dev, skinny_ns(g, dev), skinny_mn(g.M));
}

cudaError_t launch_skinny(const Gemm& g, const CUtensorMap& tB, const CUtensorMap& tA, void* ws,
                          const DeviceInfo& dev, int* dev_err, cudaStream_t s) {
  if (g.dtype == CMPX_F16)
    return g.b_kmajor ? launch_sk_mn<0, true>(g, tB, tA, ws, dev, dev_err, s)
                      : launch_sk_mn<0, false>(g, tB, tA, ws, dev, dev_err, s);
  return g.b_kmajor ? launch_sk_mn<1, true>(g, tB, tA, ws, dev, dev_err, s)
                    : launch_sk_mn<1, false>(g, tB, tA, ws, dev, dev_err, s);
}

}  // namespace cmpx

// ---------------------------------------------------------------------------
// Allocation-free entry point (see cmpx_matmul_skinny_noalloc in cmpx.h).
//
// The scratch lives in a fixed device array of this library: counters first
// (the same fixed region layout as the library-managed workspace), then fp32
// partials for up to kNoAllocMaxSms CTAs, two slots each, one 128-column
// slab of up to 64 accumulator columns.
namespace cmpx {
namespace {

constexpr int kNoAllocMaxSms = 160;
constexpr size_t kNoAllocScratchBytes = kSkinnyCounterBytes + size_t(kNoAllocMaxSms) * 2 * 1 * 64 * 128 * 4;

// In host code this name is only a stand-in for the symbol: its device
// address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up on
// the first call per device, with that device current).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CMPX_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return CMPX_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return CMPX_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return CMPX_OK;
}

template <int FMT, bool B_KMAJOR>
cudaError_t launch_noalloc_mn(const Gemm& g, const CUtensorMap& tB, const CUtensorMap& tA, void* ws,
                              const DeviceInfo& dev, int* dev_err, cudaStream_t s) {
  switch (skinny_mn(g.M)) {
    case 16: return launch_sk_impl<FMT, B_KMAJOR, 16, 1>(g, tB, tA, ws, dev, dev_err, s);
    case 32: return launch_sk_impl<FMT, B_KMAJOR, 32, 1>(g, tB, tA, ws, dev, dev_err, s);
    default: return launch_sk_impl<FMT, B_KMAJOR, 64, 1>(g, tB, tA, ws, dev, dev_err, s);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace cmpx

extern "C" CMPX_API int cmpx_matmul_skinny_noalloc(int dtype, const void* A, const void* B, void* C,
                                                   const void* bias, int64_t M, int64_t N, int64_t K, int b_layout,
                                                   cmpx_stream_t stream) {
  using namespace cmpx;
  if (dtype != CMPX_F16 && dtype != CMPX_BF16) return CMPX_ERR_INVALID_ARG;
  if (b_layout != CMPX_B_KN && b_layout != CMPX_B_NK) return CMPX_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K < 0) return CMPX_ERR_INVALID_ARG;
  const int64_t tiles = (N + 127) / 128;
  if (M > 64 || tiles > kSkinnyMaxTiles || K > (int64_t(1) << 31) - 1) return CMPX_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return CMPX_OK;
  if (C == nullptr || (K > 0 && (A == nullptr || B == nullptr))) return CMPX_ERR_INVALID_ARG;
  if (K == 0) return CMPX_ERR_UNSUPPORTED;  // nothing to reduce; use cmpx_gemm
  if (!al16(A) || !al16(B) || !al16(C) || (K * 2) % 16 != 0 || (N * 2) % 16 != 0) return CMPX_ERR_UNSUPPORTED;

  DeviceInfo dev{};
  int* err_word = nullptr;
  int st = device_facts(&dev, &err_word);
  if (st != CMPX_OK) return st;
  if (dev.num_sms > kNoAllocMaxSms) return CMPX_ERR_TOO_LARGE;
  void* ws = nullptr;
  if ((st = noalloc_scratch(&ws)) != CMPX_OK) return st;

  Gemm g{};
  g.dtype = dtype;
  g.A = A;
  g.B = B;
  g.C = C;
  g.bias = bias;
  g.batch = 1;
  g.M = M;
  g.N = N;
  g.K = K;
  g.lda = K;
  g.ldb = b_layout == CMPX_B_KN ? N : K;
  g.ldc = N;
  g.sa = M * K;
  g.sb = N * K;
  g.sc = M * N;
  g.b_kmajor = b_layout == CMPX_B_NK ? 1 : 0;

  CUtensorMap tB, tA;
  st = g.b_kmajor ? encode_tmap_3d(&tB, dtype, B, K, N, 1, K, g.sb, 64, 128)
                  : encode_tmap_3d(&tB, dtype, B, N, K, 1, N, g.sb, 64, 128);
  if (st != CMPX_OK) return st;
  st = encode_tmap_3d(&tA, dtype, A, K, M, 1, K, g.sa, 64, uint32_t(skinny_mn(M)));
  if (st != CMPX_OK) return st;

  // Counters must start at zero; a call that was cut short could have left
  // some behind, so clear the ones this call uses.
  if (cudaMemsetAsync(ws, 0, size_t(tiles) * 4 * sizeof(int), stream) != cudaSuccess) return CMPX_ERR_CUDA;
  cudaError_t e;
  if (dtype == CMPX_F16)
    e = g.b_kmajor ? launch_noalloc_mn<0, true>(g, tB, tA, ws, dev, err_word, stream)
                   : launch_noalloc_mn<0, false>(g, tB, tA, ws, dev, err_word, stream);
  else
    e = g.b_kmajor ? launch_noalloc_mn<1, true>(g, tB, tA, ws, dev, err_word, stream)
                   : launch_noalloc_mn<1, false>(g, tB, tA, ws, dev, err_word, stream);
  return e == cudaSuccess ? CMPX_OK : CMPX_ERR_CUDA;
}
