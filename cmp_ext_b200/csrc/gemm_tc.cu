// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// Replaces the reference's SIMT tile kernels gemm_fp16_ampere_optimized_v3
// (src/cuda/fp16_matmul.cu:63-283), gemm_bf16_kernel
// (src/cuda/bf16_matmul.cu:51-226) and gemm_fp32_ga100_kernel
// (src/cuda/fp32_matmul.cu:31-184).  Same product C = A*B over row-major
// operands; the arithmetic differs on purpose: fp32 accumulation in TMEM
// (fp16/bf16) and 3xTF32 (fp32), both more accurate than the reference's
// half-precision / FMA-free accumulation.
//
// CTA layout (192 threads, one CTA per SM, grid = min(tiles, #SMs)):
//   warp 0      TMA producer: fills a STAGES-deep ring of A/B tiles
//   warp 1      TMEM allocator + MMA issuer (one thread)
//   warps 2..5  epilogue: TMEM -> registers -> (+bias) -> global
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap
// the main loop of tile i+1.  Tiles are visited in grouped-M order so the A
// row-panels and B column-panels of the ~148 tiles in flight stay in L2.
//
// Shared-memory operand layouts (128-byte swizzle, written by TMA):
//   A tile [128 rows][128 B of K]           K-major, SBO = 1024
//   B tile, [K,N] source: BN/CW chunks of [BK rows][128 B of N], MN-major,
//           LBO = chunk bytes, SBO = 1024   (CW = 128 B / elem)
//   B tile, [N,K] source: [BN rows][128 B of K], K-major, SBO = 1024
#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "ptx.cuh"

namespace cmpx {
namespace {

struct TcParams {
  void* C;
  const void* bias;
  int M, N, K, batch;
  long long ldc, stride_c;
  int tiles_m, tiles_n, group_m;
  int a_bcast;
  int bias_m;
  PeerOut peers;
  int* err;
};

// FMT: 0 = f16, 1 = bf16, 2 = tf32x3 (fp32 in/out, tf32 hi/lo operands),
//      3 = bf16x3 (fp32 in/out, bf16 hi/lo operands), 4 = bf16x3 with the
//      two hi-A products in one MMA of width 2*BN (see below)
template <int FMT, bool B_KMAJOR, int BN_, int STAGES_>
struct TcCfg {
  static constexpr bool SPLIT = FMT >= 2;     // fp32 product from hi/lo operand splits
  static constexpr int E = FMT == 2 ? 4 : 2;  // operand element bytes in shared memory
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  static constexpr int BK = 128 / E;         // one 128-byte swizzle atom of K
  static constexpr int NOPS = SPLIT ? 2 : 1;  // hi (+ lo) copies per operand
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = NOPS * (A_BYTES + B_BYTES);
  static constexpr int CW = 128 / E;         // N-major chunk width in elements
  static constexpr int CHUNK_BYTES = BK * 128;
  static constexpr int KSTEP_BYTES_MN = (32 / E) * 128;  // UMMA_K rows of an MN-major tile
  // TMEM accumulator buffers.  fp16/bf16: two (epilogue of tile i overlaps
  // the main loop of tile i+1), one per tile.  Split formats: the tensor
  // core's fp32 accumulation over long MMA chains drifts (its rounding is
  // biased), so the K loop is cut into chunks of KCH k-blocks (128 elements of
  // K), each summed afresh in TMEM and added into fp32 registers by the
  // epilogue with IEEE round-to-nearest; four buffers let the MMA run three
  // chunks ahead.
  // FMT 4 issues Ah*[Bh | Bl] as one MMA of width 2*BN (B's hi and lo
  // blocks are adjacent K-major rows in shared memory), then Al*Bh into the
  // first half: two accumulator halves per tile that the epilogue adds.
  static constexpr bool NCAT = FMT == 4;
  static constexpr int ACC_COLS = NCAT ? 2 * BN : BN;
  // 3xTF32 with 256-column tiles: two 256-column chunk buffers fill TMEM, and
  // two groups of four epilogue warps each keep 128 of a row's columns in
  // registers (one thread per row would need 256 accumulator registers).
  static constexpr int EPI_GROUPS = (FMT == 2 && BN == 256) ? 2 : 1;
  static constexpr int THREADS = 64 + 128 * EPI_GROUPS;
  static constexpr int NACC = NCAT ? 2 : SPLIT ? (EPI_GROUPS == 2 ? 2 : 4) : 2;
  static constexpr int KCH = SPLIT ? 128 / BK : (1 << 30);
  static constexpr uint32_t TMEM_COLS = NACC * ACC_COLS;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + 1024 + 512;
  // operand formats: 0 = f16, 1 = bf16 (kind::f16), 2 = tf32 (kind::tf32)
  static constexpr uint32_t IDESC =
      make_idesc(FMT == 2 ? 2u : FMT == 0 ? 0u : 1u, 0u, B_KMAJOR ? 0u : 1u, BM, NCAT ? 2 * BN : BN);
  static constexpr uint32_t IDESC_HALF = make_idesc(1u, 0u, B_KMAJOR ? 0u : 1u, BM, BN);  // FMT 4: Al*Bh
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
  static_assert(B_KMAJOR || BN % CW == 0, "BN must be whole N-major chunks");
  // An MN-major tf32 operand needs the 128B swizzle with 32B atoms; the
  // split pre-pass stores fp32 B K-major instead, so that form is not built.
  // bf16 splits of a [K,N] B stay N-major (the 16-bit MN-major layout above;
  // for FMT 4 the lo chunks follow the hi chunks at the same LBO, so hi|lo
  // is one operand of width 2*BN).
  static_assert(FMT != 2 || B_KMAJOR, "3xTF32 takes B K-major");
};

__device__ __forceinline__ void decode_tile(int t, const TcParams& p, int& b, int& tm, int& tn) {
  const int per_batch = p.tiles_m * p.tiles_n;
  b = t / per_batch;
  const int r = t - b * per_batch;
  const int gw = p.group_m * p.tiles_n;
  const int g = r / gw;
  const int first_m = g * p.group_m;
  const int gm = min(p.tiles_m - first_m, p.group_m);
  const int rr = r - g * gw;
  tm = first_m + rr % gm;
  tn = rr / gm;
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
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Stores 32 consecutive fp32 accumulator columns of one output row.
// Full 16-byte groups inside [0, N) use vector stores; a ragged last group
// falls back to scalar stores.
template <typename T>
__device__ __forceinline__ void store_row32(T* crow, const T* bias, float rowb, int col0, int N,
                                            const uint32_t (&r)[32], const PeerOut& po, size_t off) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + rowb;
  if (bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int c = col0 + i;
      if (c < N) v[i] += to_f32<T>(bias[c]);
    }
  }
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int c = col0 + g * 8;
      if (c + 8 <= N) {
        uint4 q;
        q.x = pack2(v[g * 8 + 0], v[g * 8 + 1], (T*)nullptr);
        q.y = pack2(v[g * 8 + 2], v[g * 8 + 3], (T*)nullptr);
        q.z = pack2(v[g * 8 + 4], v[g * 8 + 5], (T*)nullptr);
        q.w = pack2(v[g * 8 + 6], v[g * 8 + 7], (T*)nullptr);
        *reinterpret_cast<uint4*>(crow + c) = q;
        for (int pi = 0; pi < po.n; ++pi) *reinterpret_cast<uint4*>(static_cast<T*>(po.base[pi]) + off + c) = q;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (c + i < N) {
            T h;
            if constexpr (std::is_same<T, __half>::value)
              h = __float2half_rn(v[g * 8 + i]);
            else
              h = __float2bfloat16_rn(v[g * 8 + i]);
            crow[c + i] = h;
            for (int pi = 0; pi < po.n; ++pi) static_cast<T*>(po.base[pi])[off + c + i] = h;
          }
      }
    }
  } else {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const int c = col0 + g * 4;
      if (c + 4 <= N) {
        const float4 f = make_float4(v[g * 4], v[g * 4 + 1], v[g * 4 + 2], v[g * 4 + 3]);
        *reinterpret_cast<float4*>(crow + c) = f;
        for (int pi = 0; pi < po.n; ++pi) *reinterpret_cast<float4*>(static_cast<T*>(po.base[pi]) + off + c) = f;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (c + i < N) {
            crow[c + i] = v[g * 4 + i];
            for (int pi = 0; pi < po.n; ++pi) static_cast<T*>(po.base[pi])[off + c + i] = v[g * 4 + i];
          }
      }
    }
  }
}

template <int FMT, bool B_KMAJOR, int BN, int STAGES>
__global__ void __launch_bounds__(TcCfg<FMT, B_KMAJOR, BN, STAGES>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                   const TcParams p) {
  using Cfg = TcCfg<FMT, B_KMAJOR, BN, STAGES>;
  using OutT = typename std::conditional<FMT == 0, __half, typename std::conditional<FMT == 1, __nv_bfloat16, float>::type>::type;  // split formats: fp32

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + size_t(STAGES) * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;      // [NACC]
  uint64_t* acc_empty = acc_full + Cfg::NACC;   // [NACC]
  uint64_t* drain_bar = acc_empty + Cfg::NACC;  // [1]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < Cfg::NACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128 * Cfg::EPI_GROUPS);
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

  const int total_tiles = p.tiles_m * p.tiles_n * p.batch;
  const int num_kb = (p.K + Cfg::BK - 1) / Cfg::BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      if (Cfg::SPLIT) {
        prefetch_tmap(&tmA2);
        prefetch_tmap(&tmB2);
      }
      uint32_t stage = 0, phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        int b, tm, tn;
        decode_tile(t, p, b, tm, tn);
        const int m0 = tm * Cfg::BM, n0 = tn * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            record_error(p.err, abort_flag, kDevTimeoutEmpty);
            ok = false;
            break;
          }
          uint8_t* sA = smem + size_t(stage) * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::NOPS * Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          const int k0 = kb * Cfg::BK;
          const int za = p.a_bcast ? 0 : b;
          tma_load_3d(sA, &tmA, &full_bar[stage], k0, m0, za);
          if (Cfg::SPLIT) tma_load_3d(sA + Cfg::A_BYTES, &tmA2, &full_bar[stage], k0, m0, za);
          if (B_KMAJOR) {
            tma_load_3d(sB, &tmB, &full_bar[stage], k0, n0, b);
            if (Cfg::SPLIT) tma_load_3d(sB + Cfg::B_BYTES, &tmB2, &full_bar[stage], k0, n0, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / Cfg::CW; ++j) {
              tma_load_3d(sB + j * Cfg::CHUNK_BYTES, &tmB, &full_bar[stage], n0 + j * Cfg::CW, k0, b);
              if (Cfg::SPLIT)
                tma_load_3d(sB + Cfg::B_BYTES + j * Cfg::CHUNK_BYTES, &tmB2, &full_bar[stage], n0 + j * Cfg::CW,
                            k0, b);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits.
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
      uint32_t cc = 0;  // accumulator chunks issued by this CTA
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        for (int kc = 0; kc < num_kb && ok; kc += Cfg::KCH, ++cc) {
          const int acc = int(cc % Cfg::NACC);
          const uint32_t acc_phase = (cc / Cfg::NACC) & 1;
          if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag)) {
            record_error(p.err, abort_flag, kDevTimeoutAccEmpty);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + uint32_t(acc * Cfg::ACC_COLS);
          const int kend = min(num_kb, kc + Cfg::KCH);
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
              record_error(p.err, abort_flag, kDevTimeoutFull);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + size_t(stage) * Cfg::STAGE_BYTES);
            const uint32_t b_addr = a_addr + Cfg::NOPS * Cfg::A_BYTES;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t adesc = make_sdesc_sw128(a_addr + ks * 32, 16, 1024);
              const uint64_t bdesc = B_KMAJOR ? make_sdesc_sw128(b_addr + ks * 32, 16, 1024)
                                              : make_sdesc_sw128(b_addr + ks * Cfg::KSTEP_BYTES_MN,
                                                                 Cfg::CHUNK_BYTES, 1024);
              const uint32_t accum = (kb != kc || ks != 0) ? 1u : 0u;
              if constexpr (Cfg::SPLIT) {
                const uint64_t adesc_lo = make_sdesc_sw128(a_addr + Cfg::A_BYTES + ks * 32, 16, 1024);
                const uint64_t bdesc_lo =
                    B_KMAJOR ? make_sdesc_sw128(b_addr + Cfg::B_BYTES + ks * 32, 16, 1024)
                             : make_sdesc_sw128(b_addr + Cfg::B_BYTES + ks * Cfg::KSTEP_BYTES_MN, Cfg::CHUNK_BYTES, 1024);
                // small cross terms first, then the dominant hi*hi product
                if constexpr (FMT == 2) {
                  mma_tf32(d_tmem, adesc_lo, bdesc, Cfg::IDESC, accum);
                  mma_tf32(d_tmem, adesc, bdesc_lo, Cfg::IDESC, 1u);
                  mma_tf32(d_tmem, adesc, bdesc, Cfg::IDESC, 1u);
                } else if constexpr (Cfg::NCAT) {
                  (void)bdesc_lo;
                  mma_f16(d_tmem, adesc, bdesc, Cfg::IDESC, accum);         // [Ah*Bh | Ah*Bl]
                  mma_f16(d_tmem, adesc_lo, bdesc, Cfg::IDESC_HALF, 1u);    // + Al*Bh
                } else {
                  mma_f16(d_tmem, adesc_lo, bdesc, Cfg::IDESC, accum);
                  mma_f16(d_tmem, adesc, bdesc_lo, Cfg::IDESC, 1u);
                  mma_f16(d_tmem, adesc, bdesc, Cfg::IDESC, 1u);
                }
              } else {
                mma_f16(d_tmem, adesc, bdesc, Cfg::IDESC, accum);
              }
            }
            mma_commit(&empty_bar[stage]);  // frees the smem slot once these MMAs retire
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (ok) mma_commit(&acc_full[acc]);  // chunk ready for the epilogue
        }
      }
      if (!ok) {
        // Wait for MMAs in flight before TMEM is released.
        mma_commit(drain_bar);
        volatile int never = 0;
        mbar_wait(drain_bar, 0, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    OutT* C = reinterpret_cast<OutT*>(p.C);
    const OutT* bias = reinterpret_cast<const OutT*>(p.bias);
    uint32_t cc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      int b, tm, tn;
      decode_tile(t, p, b, tm, tn);
      const int row = tm * Cfg::BM + q * 32 + lane;
      const size_t row_off = size_t(b) * p.stride_c + size_t(row) * p.ldc;
      OutT* crow = C + row_off;
      const OutT* colb = p.bias_m ? nullptr : bias;
      const float rowb = (p.bias_m && bias != nullptr && row < p.M) ? to_f32<OutT>(bias[row]) : 0.0f;
      if constexpr (Cfg::SPLIT) {
        // Sum the tile's chunks in registers (IEEE fp32 adds), then store.
        // this thread's share: columns [h * RC, (h + 1) * RC) of the tile
        constexpr int RC = BN / Cfg::EPI_GROUPS;
        const int h = Cfg::EPI_GROUPS == 1 ? 0 : (warp - 2) >> 2;
        float racc[RC];
#pragma unroll
        for (int i = 0; i < RC; ++i) racc[i] = 0.0f;
        for (int kc = 0; kc < num_kb; kc += Cfg::KCH, ++cc) {
          const int acc = int(cc % Cfg::NACC);
          const uint32_t acc_phase = (cc / Cfg::NACC) & 1;
          ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, abort_flag));
          if (!ok) {
            if (lane == 0) record_error(p.err, abort_flag, kDevTimeoutAccFull);
            break;
          }
          tc_fence_after();
          const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * Cfg::ACC_COLS);
#pragma unroll
          for (int cc2 = 0; cc2 < Cfg::ACC_COLS / 32 / Cfg::EPI_GROUPS; ++cc2) {
            const int c = h * (RC / 32) + cc2;
            const int o = (c * 32) % BN - h * RC;  // FMT 4: the second half adds onto the same columns
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {  // 16 columns at a time keeps the register count down
              uint32_t r[16];
              tmem_ld_32x32b_x16(t_row + c * 32 + hh * 16, r);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i)
                racc[o + hh * 16 + i] = __fadd_rn(racc[o + hh * 16 + i], __uint_as_float(r[i]));
            }
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[acc]);
        }
        if (!ok) break;
        if (row < p.M) {
#pragma unroll
          for (int c = 0; c < RC / 32; ++c) {
            uint32_t r[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(racc[c * 32 + i]);
            store_row32<OutT>(crow, colb, rowb, tn * BN + h * RC + c * 32, p.N, r, p.peers, row_off);
          }
        }
      } else {
        const int acc = int(cc % Cfg::NACC);
        const uint32_t acc_phase = (cc / Cfg::NACC) & 1;
        ++cc;
        // warp-uniform decision: every lane must take part in tcgen05.ld
        ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, abort_flag));
        if (!ok) {
          if (lane == 0) record_error(p.err, abort_flag, kDevTimeoutAccFull);
          break;
        }
        tc_fence_after();
        const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait();
          if (row < p.M) store_row32<OutT>(crow, colb, rowb, tn * BN + c * 32, p.N, r, p.peers, row_off);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
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

template <int FMT, bool B_KMAJOR, int BN, int STAGES>
cudaError_t launch_tc_impl(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tA2,
                           const CUtensorMap& tB2, const DeviceInfo& dev, int* dev_err, cudaStream_t s) {
  using Cfg = TcCfg<FMT, B_KMAJOR, BN, STAGES>;
  auto kern = gemm_tc_kernel<FMT, B_KMAJOR, BN, STAGES>;
  static_assert(Cfg::SMEM <= 232448, "shared memory budget");
  static unsigned long long smem_set = 0;  // one flag word per kernel instantiation
  cudaError_t e = set_smem_once(kern, int(Cfg::SMEM), smem_set);
  if (e != cudaSuccess) return e;
  TcParams p;
  p.C = g.C;
  p.bias = g.bias;
  p.M = int(g.M);
  p.N = int(g.N);
  p.K = int(g.K);
  p.batch = int(g.batch);
  p.ldc = g.ldc;
  p.stride_c = g.sc;
  p.tiles_m = int((g.M + Cfg::BM - 1) / Cfg::BM);
  p.tiles_n = int((g.N + BN - 1) / BN);
  p.group_m = 16;
  p.a_bcast = g.a_bcast;
  p.bias_m = g.bias_m;
  p.peers = g.peers;
  p.err = dev_err;
  const long long total = 1LL * p.tiles_m * p.tiles_n * p.batch;
  const int grid = int(total < dev.num_sms ? total : dev.num_sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  apply_pdl(cfg, attr, 0);
  return cudaLaunchKernelEx(&cfg, kern, tA, tB, tA2, tB2, p);
}

}  // namespace

cudaError_t launch_tc_f16(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tB, int bn, const DeviceInfo& dev,
                          int* dev_err, cudaStream_t s) {
  (void)bn;
  if (g.dtype == CMPX_F16) {
    if (g.b_kmajor) return launch_tc_impl<0, true, 256, 4>(g, tA, tB, tA, tB, dev, dev_err, s);
    return launch_tc_impl<0, false, 256, 4>(g, tA, tB, tA, tB, dev, dev_err, s);
  }
  if (g.b_kmajor) return launch_tc_impl<1, true, 256, 4>(g, tA, tB, tA, tB, dev, dev_err, s);
  return launch_tc_impl<1, false, 256, 4>(g, tA, tB, tA, tB, dev, dev_err, s);
}

cudaError_t launch_tc_tf32x3(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tA2, const CUtensorMap& tB,
                             const CUtensorMap& tB2, const DeviceInfo& dev, int* dev_err, cudaStream_t s) {
  if (tf32x3_block_n() == 256) return launch_tc_impl<2, true, 256, 2>(g, tA, tB, tA2, tB2, dev, dev_err, s);
  return launch_tc_impl<2, true, 128, 3>(g, tA, tB, tA2, tB2, dev, dev_err, s);
}

cudaError_t launch_tc_bf16x3(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tA2, const CUtensorMap& tB,
                             const CUtensorMap& tB2, bool b_nmajor, const DeviceInfo& dev, int* dev_err,
                             cudaStream_t s) {
  static int ncat = -1;
  if (ncat < 0) {
    // Measured on a B200 (8192^3, isolated launches): 2.90 ms with the
    // width-2*BN form against 2.99 ms with three width-BN MMAs, at a lower
    // power-capped clock; CMPX_BF16X3_NCAT=0 selects the three-MMA form.
    const char* e = std::getenv("CMPX_BF16X3_NCAT");
    ncat = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  if (b_nmajor) {
    if (ncat) return launch_tc_impl<4, false, 128, 3>(g, tA, tB, tA2, tB2, dev, dev_err, s);
    return launch_tc_impl<3, false, 128, 3>(g, tA, tB, tA2, tB2, dev, dev_err, s);
  }
  if (ncat) return launch_tc_impl<4, true, 128, 3>(g, tA, tB, tA2, tB2, dev, dev_err, s);
  return launch_tc_impl<3, true, 128, 3>(g, tA, tB, tA2, tB2, dev, dev_err, s);
}

// ------------------------------------------------------------------ split
// fp32 X -> hi + lo with hi = round(x), lo = round(x - hi), in one of two
// operand formats: tf32 (kept in fp32 containers, cvt.rna) for 3xTF32, or
// bf16 (round-to-nearest-even) for bf16x3.  hi*hi + hi*lo + lo*hi then
// recovers the product to about 2^-21 (tf32) or 2^-16 (bf16) relative.
namespace {
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi is rounded to nearest, so a finite x within half an ulp of the format's
// largest finite value would round hi to infinity (and lo to -infinity),
// where the reference's fp32 arithmetic stays finite.  hi is then clamped to
// the largest finite value of the format, with x's sign, and lo carries the
// (small, exactly representable) rest.
__device__ __forceinline__ void split1(float x, float& h, float& l) {
  h = tf32_rna(x);
  if (isinf(h) && !isinf(x)) h = copysignf(__uint_as_float(0x7F7FE000u), x);  // largest finite tf32
  l = tf32_rna(x - h);
}
__device__ __forceinline__ void split1(float x, __nv_bfloat16& h, __nv_bfloat16& l) {
  h = __float2bfloat16_rn(x);
  if (__hisinf(h) && !isinf(x)) h = __ushort_as_bfloat16(x < 0.0f ? 0xFF7Fu : 0x7F7Fu);  // largest finite bf16
  l = __float2bfloat16_rn(x - __bfloat162float(h));
}

// Four consecutive split values as one 16-byte (tf32) or 8-byte (bf16) store.
template <typename S>
struct Vec4;
template <>
struct Vec4<float> {
  float4 v;
  __device__ __forceinline__ void set(int i, float x) { (&v.x)[i] = x; }
  __device__ __forceinline__ void store(float* p) const { __stcs(reinterpret_cast<float4*>(p), v); }
};
template <>
struct Vec4<__nv_bfloat16> {
  __nv_bfloat16 v[4];
  __device__ __forceinline__ void set(int i, __nv_bfloat16 x) { v[i] = x; }
  __device__ __forceinline__ void store(__nv_bfloat16* p) const {
    uint2 u;
    u.x = uint32_t(__bfloat16_as_ushort(v[0])) | (uint32_t(__bfloat16_as_ushort(v[1])) << 16);
    u.y = uint32_t(__bfloat16_as_ushort(v[2])) | (uint32_t(__bfloat16_as_ushort(v[3])) << 16);
    __stcs(reinterpret_cast<uint2*>(p), u);
  }
};

// X [rows][cols] (row stride ld) -> packed hi, lo [rows][cols].  Vector
// form: cols % 4 == 0, ld % 4 == 0 and X 16-byte aligned.  A block holds
// 256 >> tpr_log2 rows of 1 << tpr_log2 threads each (a power of two >= the
// row's float4 count, at most 256), so short rows still keep every thread
// busy; blocks stride over row groups and no index needs a division.
template <typename S>
__global__ void split_vec_kernel(const float* __restrict__ X, S* __restrict__ hi, S* __restrict__ lo,
                                 long long rows, long long cols, long long ld, long long sx, int tpr_log2) {
  pdl_trigger();
  pdl_wait();  // X may be the previous kernel's output
  const long long b = blockIdx.y;
  const long long c4 = cols / 4;
  const float* xb = X + b * sx;
  S* hb = hi + b * rows * cols;
  S* lb = lo + b * rows * cols;
  const int tpr = 1 << tpr_log2;
  const int sub = threadIdx.x >> tpr_log2;
  const int lane_r = threadIdx.x & (tpr - 1);
  const long long rpb = blockDim.x >> tpr_log2;
  for (long long r = blockIdx.x * rpb + sub; r < rows; r += gridDim.x * rpb) {
    const float4* xr = reinterpret_cast<const float4*>(xb + r * ld);
    S* hr = hb + r * cols;
    S* lr = lb + r * cols;
    for (long long c = lane_r; c < c4; c += tpr) {
      const float4 x = __ldcs(xr + c);
      Vec4<S> h, l;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S hj, lj;
        split1((&x.x)[j], hj, lj);
        h.set(j, hj);
        l.set(j, lj);
      }
      h.store(hr + 4 * c);
      l.store(lr + 4 * c);
    }
  }
}

template <typename S>
__global__ void split_kernel(const float* __restrict__ X, S* __restrict__ hi, S* __restrict__ lo, long long rows,
                             long long cols, long long ld, long long sx) {
  pdl_trigger();
  pdl_wait();  // X may be the previous kernel's output
  const long long b = blockIdx.y;
  const long long n = rows * cols;
  const float* xb = X + b * sx;
  S* hb = hi + b * n;
  S* lb = lo + b * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols, c = i - r * cols;
    split1(xb[r * ld + c], hb[i], lb[i]);
  }
}

// Same split, writing the transpose ([cols][rows]) through 64x64 shared
// tiles; float4 reads along cols and 4-element vector writes along rows
// (vector form: rows % 4 == 0, cols % 4 == 0, ld % 4 == 0, X 16-byte aligned).
template <typename S>
__global__ void __launch_bounds__(256) split_transpose_kernel(const float* __restrict__ X, S* __restrict__ hi,
                                                              S* __restrict__ lo, long long rows, long long cols,
                                                              long long ld, long long sx) {
  pdl_trigger();
  pdl_wait();
  __shared__ S th[64][65];
  __shared__ S tl[64][65];
  const long long b = blockIdx.z;
  const float* xb = X + b * sx;
  S* hb = hi + b * rows * cols;
  S* lb = lo + b * rows * cols;
  const long long r0 = (long long)blockIdx.y * 64, c0 = (long long)blockIdx.x * 64;
  const int t = threadIdx.x;
#pragma unroll
  for (int it = 0; it < 4; ++it) {  // 64 rows x 16 float4
    const int e = t + it * 256;
    const int rr = e >> 4, cc = (e & 15) * 4;
    const long long r = r0 + rr, c = c0 + cc;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows && c < cols) x = __ldcs(reinterpret_cast<const float4*>(xb + r * ld + c));
#pragma unroll
    for (int j = 0; j < 4; ++j) split1((&x.x)[j], th[rr][cc + j], tl[rr][cc + j]);
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < 4; ++it) {  // 64 output rows (= input cols) x 16 vectors along input rows
    const int e = t + it * 256;
    const int cc = e >> 4, rr = (e & 15) * 4;
    const long long c = c0 + cc, r = r0 + rr;
    if (c < cols && r < rows) {
      Vec4<S> h, l;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        h.set(j, th[rr + j][cc]);
        l.set(j, tl[rr + j][cc]);
      }
      h.store(hb + c * rows + r);
      l.store(lb + c * rows + r);
    }
  }
}
}  // namespace

// 256-thread launch with the programmatic-dependent-launch attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_plain_pdl(void (*kern)(KArgs...), dim3 grid, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  apply_pdl(cfg, attr, 0);
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

namespace {
template <typename S>
cudaError_t launch_split_impl(const float* X, S* hi, S* lo, int64_t batch, int64_t rows, int64_t cols, int64_t ld,
                              int64_t sx, bool transpose, int num_sms, cudaStream_t s) {
  const bool vec = (reinterpret_cast<uintptr_t>(X) & 15u) == 0 && cols % 4 == 0 && ld % 4 == 0 &&
                   (batch <= 1 || sx % 4 == 0);
  if (transpose) {
    // The transpose is only needed for [K,N] B, whose packed copy is used by
    // the tensor-core path: K (= rows) % 4 == 0 holds there.
    if (!vec || rows % 4 != 0) return cudaErrorInvalidValue;
    const dim3 grid{unsigned((cols + 63) / 64), unsigned((rows + 63) / 64), unsigned(batch)};
    return launch_plain_pdl(split_transpose_kernel<S>, grid, s, X, hi, lo, rows, cols, ld, sx);
  }
  if (vec) {
    int tpr_log2 = 0;
    while (tpr_log2 < 8 && (1LL << tpr_log2) < cols / 4) ++tpr_log2;
    const long long rpb = 256 >> tpr_log2;
    // a block per row group, up to 8 resident 256-thread blocks per SM; grid-strided beyond that
    long long blocks = (rows + rpb - 1) / rpb;
    if (blocks > 8LL * num_sms) blocks = 8LL * num_sms;
    if (blocks < 1) blocks = 1;
    const dim3 grid{unsigned(blocks), unsigned(batch), 1u};
    return launch_plain_pdl(split_vec_kernel<S>, grid, s, X, hi, lo, rows, cols, ld, sx, tpr_log2);
  }
  const long long n = rows * cols;
  long long blocks = (n + 255) / 256;
  if (blocks > 8LL * num_sms) blocks = 8LL * num_sms;
  if (blocks < 1) blocks = 1;
  const dim3 grid{unsigned(blocks), unsigned(batch), 1u};
  return launch_plain_pdl(split_kernel<S>, grid, s, X, hi, lo, rows, cols, ld, sx);
}
}  // namespace

cudaError_t launch_split_tf32(const float* X, float* hi, float* lo, int64_t batch, int64_t rows, int64_t cols,
                              int64_t ld, int64_t sx, bool transpose, int num_sms, cudaStream_t s) {
  return launch_split_impl<float>(X, hi, lo, batch, rows, cols, ld, sx, transpose, num_sms, s);
}

cudaError_t launch_split_bf16(const float* X, void* hi, void* lo, int64_t batch, int64_t rows, int64_t cols,
                              int64_t ld, int64_t sx, bool transpose, int num_sms, cudaStream_t s) {
  return launch_split_impl<__nv_bfloat16>(X, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), batch,
                                          rows, cols, ld, sx, transpose, num_sms, s);
}

}  // namespace cmpx
