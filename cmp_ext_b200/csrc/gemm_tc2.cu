// Persistent tcgen05 GEMM on CTA pairs (cta_group::2) for fp16 / bf16.
//
// Same product and arithmetic as gemm_tc.cu (fp32 accumulation in TMEM,
// one rounding to the output type; replaces the reference's SIMT kernels
// src/cuda/fp16_matmul.cu:63-283 and src/cuda/bf16_matmul.cu:51-226), with
// the output tile computed by two SMs together:
//   * a cluster of two CTAs owns a 256 x PN tile; CTA rank r holds rows
//     [128 r, 128 r + 128) of the A tile and columns [PN/2 r, PN/2 (r+1)) of
//     the B tile in its shared memory;
//   * the leader (rank 0) issues one tcgen05.mma.cta_group::2 (M = 256,
//     N = PN, K = 16) per k-step, which reads both CTAs' shared memory and
//     writes each CTA's 128 accumulator rows into that CTA's TMEM;
//   * both CTAs load their own halves with TMA; the loads complete on the
//     leader's "full" barrier (no multicast: every byte lands in the CTA that
//     loaded it), and the leader's MMA completion is multicast to both CTAs'
//     "empty" and "accumulator full" barriers;
//   * each CTA's epilogue warps drain their own TMEM rows and report back to
//     the leader's "accumulator empty" barrier.
// Per SM this halves the B operand traffic of a 128 x PN tile, and the
// 256 x 128 pair tile gives twice as many tiles as a 128 x 256 tile for the
// same work per SM, which cuts the wave-quantisation tail on mid-size
// problems.
//
// Warp roles per CTA (192 threads): warp 0 TMA producer, warp 1 TMEM
// allocation (both CTAs) and MMA issue (leader only), warps 2..5 epilogue.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "ptx.cuh"

namespace cmpx {
namespace {

struct Tc2Params {
  void* C;
  const void* bias;
  int M, N, K, batch;
  long long ldc, stride_c;
  int tiles_m, tiles_n, group_m;  // in pair tiles (256 x PN)
  // Data-parallel + stream-K split: tiles [0, dp_tiles) are computed whole,
  // round-robin over the pairs; the k-blocks of the remaining sk_tiles tiles
  // (sk_units = sk_tiles * k-blocks) are split evenly over all pairs.
  int dp_tiles, sk_tiles;
  int sk_pairs;  // pairs sharing the stream-K units: min(pairs, sk_units), so none is empty
  long long sk_units;
  float* ws;      // [pair][slot 2][rank 2][128][PN] fp32 partials of split tiles
  int* counters;  // [sk tile][rank 2][epilogue warp 4], zero on entry and exit
  int a_bcast;
  int bias_m;
  PeerOut peers;
  void* mc_C;  // multicast address of C's layout (nullptr = none), see store_row32_16
  int* col_flags;  // progress flags per (M group of the raster, column group), nullptr = none
  int flag_tiles;     // pair-tile columns per column group
  int flag_groups_n;  // column groups
  unsigned epi_sleep_ns;  // epilogue's accumulator wait: sleep between polls (0 = spin)
  int* err;
};

// One unit of work of a pair: output tile `tile`, k-blocks [kb0, kb1).
// skt >= 0 marks a stream-K tile (its index among the split tiles).
struct WorkItem {
  int tile, kb0, kb1, skt;
};

__device__ __forceinline__ long long sk_begin(long long g, long long U, long long P) { return g * U / P; }
__device__ __forceinline__ long long sk_owner(long long u, long long U, long long P) { return ((u + 1) * P - 1) / U; }

// The item-th work item of pair `c` (false when there is none): first its
// whole data-parallel tiles, then the pieces of its stream-K unit range cut
// at tile boundaries.  Every role of both CTAs walks the same sequence.
__device__ __forceinline__ bool work_item(const Tc2Params& p, int c, int P, int num_kb, int item, WorkItem& w) {
  const int n_dp = c < p.dp_tiles ? (p.dp_tiles - c + P - 1) / P : 0;
  if (item < n_dp) {
    w.tile = c + item * P;
    w.kb0 = 0;
    w.kb1 = num_kb;
    w.skt = -1;
    return true;
  }
  if (p.sk_tiles == 0 || c >= p.sk_pairs) return false;
  const long long U = p.sk_units;
  const long long u0 = sk_begin(c, U, p.sk_pairs), u1 = sk_begin(c + 1, U, p.sk_pairs);
  const int j = item - n_dp;
  const long long s = j == 0 ? u0 : (u0 / num_kb + j) * (long long)num_kb;
  if (s >= u1) return false;
  const long long t = s / num_kb;
  const long long e = min(u1, (t + 1) * (long long)num_kb);
  w.skt = int(t);
  w.tile = p.dp_tiles + int(t);
  w.kb0 = int(s - t * num_kb);
  w.kb1 = int(e - t * num_kb);
  return true;
}

template <int FMT, bool B_KMAJOR, int PN, int STAGES_, bool TMA_OUT = false>
struct Tc2Cfg {
  static constexpr int BK = 64;                  // 128 bytes of K
  static constexpr int BH = PN / 2;              // B columns held by one CTA
  static constexpr int STAGES = STAGES_;
  static constexpr int A_BYTES = 128 * 128;      // 128 rows x 64 K x 2 B
  static constexpr int B_BYTES = BH * 128;       // BH columns x 64 K x 2 B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NACC = 512 / PN;          // TMEM accumulators per CTA
  static constexpr uint32_t TMEM_COLS = 512;
  // TMA_OUT: per epilogue warp, two 32 x 32 staging buffers (2 KB each)
  static constexpr int STAGING_BYTES = TMA_OUT ? 4 * 2 * 2048 : 0;
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + STAGING_BYTES + 1024 + 512;
  static constexpr uint32_t IDESC = make_idesc(uint32_t(FMT), 0u, B_KMAJOR ? 0u : 1u, 256, PN);
  static_assert(BH % 64 == 0, "B half must be whole 64-column chunks");
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
};

__device__ __forceinline__ void decode_tile2(int t, const Tc2Params& p, int& b, int& tm, int& tn) {
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

__device__ __forceinline__ void record_error2(int* err, volatile int* abort, int code) {
  *abort = 1;
  atomicCAS(err, 0, code);
}

template <typename T>
__device__ __forceinline__ float to_f32_2(T v);
template <>
__device__ __forceinline__ float to_f32_2<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32_2<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ uint32_t pack2_2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2_2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One 16-byte store through an NVLink multicast address: the switch writes
// it into every GPU's buffer bound to the multicast object.
__device__ __forceinline__ void multimem_st16(void* mc_addr, const uint4& q) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr),
               "f"(__uint_as_float(q.x)), "f"(__uint_as_float(q.y)), "f"(__uint_as_float(q.z)),
               "f"(__uint_as_float(q.w))
               : "memory");
}

// 32 consecutive accumulator columns of one output row -> +bias -> 16-bit
// output; full 16-byte groups inside [0, N) use vector stores.  With `mc`
// (the multicast address of C's layout; N % 8 == 0) each 16-byte group is
// written once through it instead of to C and the peer copies.
template <typename T>
__device__ __forceinline__ void store_row32_16(T* crow, const T* bias, float rowb, int col0, int N,
                                               const uint32_t (&r)[32], const PeerOut& po, size_t off,
                                               void* mc = nullptr) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + rowb;
  if (bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < N) v[i] += to_f32_2<T>(bias[col0 + i]);
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int c = col0 + g * 8;
    if (c + 8 <= N) {
      uint4 q;
      q.x = pack2_2(v[g * 8 + 0], v[g * 8 + 1], (T*)nullptr);
      q.y = pack2_2(v[g * 8 + 2], v[g * 8 + 3], (T*)nullptr);
      q.z = pack2_2(v[g * 8 + 4], v[g * 8 + 5], (T*)nullptr);
      q.w = pack2_2(v[g * 8 + 6], v[g * 8 + 7], (T*)nullptr);
      if (mc != nullptr) {
        multimem_st16(static_cast<T*>(mc) + off + c, q);
        continue;
      }
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
}

// Converts 32 accumulator columns (+ row / column bias) to packed 16-bit
// values, 4 x 16 bytes.  Columns at or beyond N get values that are never
// stored (TMA clips them).
template <typename T>
__device__ __forceinline__ void pack_row32_16(const uint32_t (&r)[32], const T* bias, float rowb, int col0, int N,
                                              uint4 (&o)[4]) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + rowb;
  if (bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < N) v[i] += to_f32_2<T>(bias[col0 + i]);
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    o[g].x = pack2_2(v[g * 8 + 0], v[g * 8 + 1], (T*)nullptr);
    o[g].y = pack2_2(v[g * 8 + 2], v[g * 8 + 3], (T*)nullptr);
    o[g].z = pack2_2(v[g * 8 + 4], v[g * 8 + 5], (T*)nullptr);
    o[g].w = pack2_2(v[g * 8 + 6], v[g * 8 + 7], (T*)nullptr);
  }
}

// STREAMK: the kernel may be given split (stream-K) tiles and carries their
// partial-sum hand-off; the default instantiation is whole tiles only, which
// keeps the split path's 128-float reduction registers out of it.
template <int FMT, bool B_KMAJOR, int PN, int STAGES, bool TMA_OUT, bool STREAMK>
__global__ void __launch_bounds__(192, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const Tc2Params p, const __grid_constant__ OutMaps om) {
  using Cfg = Tc2Cfg<FMT, B_KMAJOR, PN, STAGES, TMA_OUT>;
  using OutT = typename std::conditional<FMT == 0, __half, __nv_bfloat16>::type;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* staging = smem + size_t(STAGES) * Cfg::STAGE_BYTES;  // TMA_OUT only
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(staging + Cfg::STAGING_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + Cfg::NACC;
  uint64_t* drain_bar = acc_empty + Cfg::NACC;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // used in the leader only
      mbar_init(&empty_bar[s], 1);  // leader's MMA commit, multicast to both CTAs
    }
    for (int a = 0; a < Cfg::NACC; ++a) {
      mbar_init(&acc_full[a], 1);     // leader's MMA commit, multicast to both CTAs
      mbar_init(&acc_empty[a], 256);  // used in the leader only: both CTAs' epilogue threads
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, Cfg::TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_trigger();
  pdl_wait();

  const int num_kb = (p.K + Cfg::BK - 1) / Cfg::BK;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      WorkItem w;
      for (int item = 0; ok && work_item(p, cluster_id, num_clusters, num_kb, item, w); ++item) {
        int b, tm, tn;
        decode_tile2(w.tile, p, b, tm, tn);
        const int m0 = tm * 256 + int(rank) * 128;
        const int n0 = tn * PN + int(rank) * Cfg::BH;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag)) {
            record_error2(p.err, abort_flag, kDevTimeoutEmpty);
            ok = false;
            break;
          }
          const uint32_t full_leader = mapa_cluster(&full_bar[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          uint8_t* sA = smem + size_t(stage) * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          const int k0 = kb * Cfg::BK;
          tma_load_3d_pair(sA, &tmA, full_leader, k0, m0, p.a_bcast ? 0 : b);
          if (B_KMAJOR) {
            tma_load_3d_pair(sB, &tmB, full_leader, k0, n0, b);
          } else {
#pragma unroll
            for (int j = 0; j < Cfg::BH / 64; ++j) tma_load_3d_pair(sB + j * 8192, &tmB, full_leader, n0 + 64 * j, k0, b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Give copies already issued time to land before the CTA exits.
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      uint32_t lt = 0;
      WorkItem w;
      for (int item = 0; ok && work_item(p, cluster_id, num_clusters, num_kb, item, w); ++item, ++lt) {
        const int acc = int(lt % Cfg::NACC);
        const uint32_t acc_phase = (lt / Cfg::NACC) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag)) {
          record_error2(p.err, abort_flag, kDevTimeoutAccEmpty);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * PN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
            record_error2(p.err, abort_flag, kDevTimeoutFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + size_t(stage) * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t adesc = make_sdesc_sw128(a_addr + ks * 32, 16, 1024);
            const uint64_t bdesc = B_KMAJOR ? make_sdesc_sw128(b_addr + ks * 32, 16, 1024)
                                            : make_sdesc_sw128(b_addr + ks * 2048, 8192, 1024);
            mma_f16_pair(d_tmem, adesc, bdesc, Cfg::IDESC, (kb != w.kb0 || ks != 0) ? 1u : 0u);
          }
          mma_commit_pair_mc(&empty_bar[stage], 0x3);  // both CTAs' slots are free once these retire
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) mma_commit_pair_mc(&acc_full[acc], 0x3);
      }
      if (!ok) {
        mma_commit_pair_mc(drain_bar, 0x1);
        volatile int never = 0;
        mbar_wait(drain_bar, 0, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    OutT* C = reinterpret_cast<OutT*>(p.C);
    const OutT* bias = reinterpret_cast<const OutT*>(p.bias);
    uint32_t lt = 0;
    uint32_t chunk_seq = 0;  // TMA_OUT: chunks staged by this warp (buffer = parity)
    const long long P = p.sk_pairs;
    const long long first_skt =
        (p.sk_tiles > 0 && cluster_id < p.sk_pairs) ? sk_begin(cluster_id, p.sk_units, P) / num_kb : -1;
    WorkItem w;
    for (int item = 0; work_item(p, cluster_id, num_clusters, num_kb, item, w); ++item, ++lt) {
      int b, tm, tn;
      decode_tile2(w.tile, p, b, tm, tn);
      const int acc = int(lt % Cfg::NACC);
      const uint32_t acc_phase = (lt / Cfg::NACC) & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait_sleep(&acc_full[acc], acc_phase, abort_flag, p.epi_sleep_ns));
      if (!ok) {
        if (lane == 0) record_error2(p.err, abort_flag, kDevTimeoutAccFull);
        break;
      }
      tc_fence_after();
      const int lrow = q * 32 + lane;  // row within this CTA's 128-row half
      const int row = tm * 256 + int(rank) * 128 + lrow;
      const size_t row_off = size_t(b) * p.stride_c + size_t(row) * p.ldc;
      OutT* crow = C + row_off;
      const OutT* colb = p.bias_m ? nullptr : bias;
      const float rowb = (p.bias_m && bias != nullptr && row < p.M) ? to_f32_2<OutT>(bias[row]) : 0.0f;
      const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * PN);
      long long g_lo = 0, g_hi = 0;
      if (w.skt >= 0) {
        const long long t_u0 = (long long)w.skt * num_kb;
        g_lo = sk_owner(t_u0, p.sk_units, P);
        g_hi = sk_owner(t_u0 + num_kb - 1, p.sk_units, P);
      }
      const bool whole = !STREAMK || w.skt < 0 || g_lo == g_hi;
      float* part = nullptr;
      if (!whole) {
        const int slot = (w.skt == first_skt) ? 0 : 1;
        part = p.ws + ((size_t(cluster_id) * 2 + slot) * 2 + rank) * 128 * PN + size_t(lrow) * PN;
      }
#pragma unroll 1
      for (int c = 0; c < PN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        if (whole) {
          if constexpr (TMA_OUT) {
            // Stage the 32 x 32 chunk (row = lane, 64 B) and store it with one
            // TMA box per destination (C, then each peer copy of it).
            uint8_t* stg = staging + q * 4096 + (chunk_seq & 1) * 2048;
            if (lane == 0) bulk_wait_read1();  // the store that last read this buffer is done with it
            __syncwarp();
            uint4 o[4];
            pack_row32_16<OutT>(r, colb, rowb, tn * PN + c * 32, p.N, o);
#pragma unroll
            for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(stg + lane * 64 + j * 16) = o[j];
            fence_proxy_async_smem();
            __syncwarp();
            const int row0 = tm * 256 + int(rank) * 128 + q * 32;
            if (p.mc_C != nullptr) {
              // Multicast output: read the staged chunk back so that each
              // instruction writes 8 rows x 64 contiguous bytes (4 lanes per
              // row) through the multicast address, instead of 32 scattered
              // 16-byte pieces.
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int rr = i * 8 + (lane >> 2), piece = lane & 3;
                const int orow = row0 + rr, ocol = tn * PN + c * 32 + piece * 8;
                if (orow < p.M && ocol < p.N) {
                  const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 64 + piece * 16);
                  multimem_st16(static_cast<OutT*>(p.mc_C) + size_t(b) * p.stride_c + size_t(orow) * p.ldc + ocol, v);
                }
              }
              __syncwarp();  // the buffer is read before it is staged again
            } else if (lane == 0) {
              for (int d = 0; d < om.n; ++d) tma_store_3d(&om.m[d], stg, tn * PN + c * 32, row0, b);
              bulk_commit();
            }
            ++chunk_seq;
          } else {
            if (row < p.M)
              store_row32_16<OutT>(crow, colb, rowb, tn * PN + c * 32, p.N, r, p.peers, row_off, p.mc_C);
          }
        } else {
          float4* dst = reinterpret_cast<float4*>(part + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            __stcg(dst + i, make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                        __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])));
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(mapa_cluster(&acc_empty[acc], 0));
      if (p.col_flags != nullptr && whole) {
        // This warp's 32 rows of the tile are stored: one lane publishes them
        // at system scope and counts them (8 arrivals per pair tile: 4
        // epilogue warps x 2 CTAs), so a copy engine waiting on the flag
        // reads finished rows.  Per warp, so no warp ever waits on another.
        __syncwarp();
        if (lane == 0) {
          __threadfence_system();
          atomicAdd(p.col_flags + (tm / p.group_m) * p.flag_groups_n + tn / p.flag_tiles, 1);
        }
      }

      if (STREAMK && !whole) {
        // The last part of this split tile to arrive (per CTA half and
        // epilogue warp) sums the parts in pair order, adds the bias, rounds
        // once and stores; it then zeroes the counter for the next launch.
        __threadfence();
        __syncwarp();
        int prev = 0;
        int* ctr = p.counters + (size_t(w.skt) * 2 + rank) * 4 + q;
        if (lane == 0) prev = atomicAdd(ctr, 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == int(g_hi - g_lo)) {
          __threadfence();
          // Two halves of the row; per half and part, all 16 float4 loads are
          // issued before any is used (memory-level parallelism).
#pragma unroll 1
          for (int h = 0; h < PN / 128; ++h) {
            float sum[128];
#pragma unroll
            for (int i = 0; i < 128; ++i) sum[i] = 0.0f;
            for (long long gg = g_lo; gg <= g_hi; ++gg) {
              const int sl = (w.skt == sk_begin(gg, p.sk_units, P) / num_kb) ? 0 : 1;
              const float4* src = reinterpret_cast<const float4*>(
                  p.ws + ((size_t(gg) * 2 + sl) * 2 + rank) * 128 * PN + size_t(lrow) * PN + h * 128);
              float4 v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = __ldcg(src + i);
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                sum[4 * i] += v[i].x;
                sum[4 * i + 1] += v[i].y;
                sum[4 * i + 2] += v[i].z;
                sum[4 * i + 3] += v[i].w;
              }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(sum[c * 32 + i]);
              if (row < p.M)
                store_row32_16<OutT>(crow, colb, rowb, tn * PN + h * 128 + c * 32, p.N, r, p.peers, row_off, p.mc_C);
            }
          }
          if (lane == 0) *ctr = 0;
        }
      }
    }
  }

  if constexpr (TMA_OUT) {
    if (warp >= 2 && lane == 0) bulk_wait_all();  // staged output stores have landed
  }
  if (p.col_flags != nullptr && threadIdx.x == 0 && *abort_flag) {
    // A launch that gave up never completes its tiles: release every waiter
    // on the flags (the error word tells the host the output is not valid).
    const int groups = ((p.tiles_m + p.group_m - 1) / p.group_m) * p.flag_groups_n;
    for (int j = 0; j < groups; ++j) atomicAdd(p.col_flags + j, 1 << 24);
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int FMT, bool B_KMAJOR, int PN, int STAGES, bool TMA_OUT, bool STREAMK>
cudaError_t launch_tc2_run(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tB, void* ws,
                           const DeviceInfo& dev, int* dev_err, cudaStream_t s, const OutMaps& om) {
  using Cfg = Tc2Cfg<FMT, B_KMAJOR, PN, STAGES, TMA_OUT>;
  auto kern = gemm_tc2_kernel<FMT, B_KMAJOR, PN, STAGES, TMA_OUT, STREAMK>;
  static_assert(Cfg::SMEM <= 232448, "shared memory budget");
  static unsigned long long smem_set = 0;  // one flag word per kernel instantiation
  cudaError_t e = set_smem_once(kern, int(Cfg::SMEM), smem_set);
  if (e != cudaSuccess) return e;
  Tc2Params p;
  p.C = g.C;
  p.bias = g.bias;
  p.M = int(g.M);
  p.N = int(g.N);
  p.K = int(g.K);
  p.batch = int(g.batch);
  p.ldc = g.ldc;
  p.stride_c = g.sc;
  p.tiles_m = int((g.M + 255) / 256);
  p.tiles_n = int((g.N + PN - 1) / PN);
  p.group_m = tc2_group_m();
  p.a_bcast = g.a_bcast;
  p.bias_m = g.bias_m;
  p.peers = g.peers;
  p.mc_C = g.mc_C;
  p.col_flags = g.col_flags;
  p.flag_tiles = g.flag_tiles > 0 ? g.flag_tiles : 1;
  p.flag_groups_n = (p.tiles_n + p.flag_tiles - 1) / p.flag_tiles;
  p.epi_sleep_ns = epilogue_sleep_ns();
  p.err = dev_err;
  const long long total = 1LL * p.tiles_m * p.tiles_n * p.batch;
  const long long pairs = dev.num_sms / 2;
  const int num_kb = int((g.K + Cfg::BK - 1) / Cfg::BK);
  // Stream-K region: the last, partial wave plus one full wave before it (so
  // each split tile has only two or three parts), or everything when there
  // is less than a wave.
  const long long rem = total % pairs;
  long long sk = 0;
  if (STREAMK && ws != nullptr && rem != 0) sk = total >= pairs ? rem + pairs : total;
  p.dp_tiles = int(total - sk);
  p.sk_tiles = int(sk);
  p.sk_units = sk * num_kb;
  p.sk_pairs = int(p.sk_units < pairs ? p.sk_units : pairs);
  p.counters = reinterpret_cast<int*>(ws);
  p.ws = ws != nullptr ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kSkinnyCounterBytes) : nullptr;
  const long long clusters = sk > 0 ? pairs : (total < pairs ? total : pairs);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(2 * clusters), 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  apply_pdl(cfg, attr, 1);
  e = cudaLaunchKernelEx(&cfg, kern, tA, tB, p, om);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int FMT, bool B_KMAJOR, int PN, int STAGES>
cudaError_t launch_tc2_impl(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tB, void* ws,
                            const DeviceInfo& dev, int* dev_err, cudaStream_t s, const OutMaps* om) {
  // Peer outputs (staged TMA stores) run whole tiles only.
  if (om != nullptr) return launch_tc2_run<FMT, B_KMAJOR, PN, STAGES, true, false>(g, tA, tB, nullptr, dev, dev_err, s, *om);
  // Multicast output: the staged epilogue with no TMA store maps.
  static OutMaps none_mc{};
  if (g.mc_C != nullptr)
    return launch_tc2_run<FMT, B_KMAJOR, PN, STAGES, true, false>(g, tA, tB, nullptr, dev, dev_err, s, none_mc);
  static OutMaps none{};
  if (ws != nullptr) return launch_tc2_run<FMT, B_KMAJOR, PN, STAGES, false, true>(g, tA, tB, ws, dev, dev_err, s, none);
  return launch_tc2_run<FMT, B_KMAJOR, PN, STAGES, false, false>(g, tA, tB, nullptr, dev, dev_err, s, none);
}

}  // namespace

// Pair-tile width: 256 x 128 (twice the tiles, for fewer-wave problems) by
// default; the B half held per CTA is pair_n / 2 columns.
// Workspace for the stream-K part (0 when the tiles fill whole waves): the
// shared fixed counter region, then [pair][2 slots][2 ranks][128][pair_n] fp32.
size_t tc2_workspace_bytes(const Gemm& g, int pair_n, const DeviceInfo& dev) {
  const long long pairs = dev.num_sms / 2;
  const long long total = g.batch * ((g.M + 255) / 256) * ((g.N + pair_n - 1) / pair_n);
  if (total % pairs == 0) return 0;
  return kSkinnyCounterBytes + size_t(pairs) * 2 * 2 * 128 * size_t(pair_n) * 4;
}

cudaError_t launch_tc2_f16(const Gemm& g, const CUtensorMap& tA, const CUtensorMap& tB, int pair_n, void* ws,
                           const DeviceInfo& dev, int* dev_err, cudaStream_t s, const OutMaps* om) {
  if (pair_n == 256) {
    if (g.dtype == CMPX_F16)
      return g.b_kmajor ? launch_tc2_impl<0, true, 256, 6>(g, tA, tB, ws, dev, dev_err, s, om)
                        : launch_tc2_impl<0, false, 256, 6>(g, tA, tB, ws, dev, dev_err, s, om);
    return g.b_kmajor ? launch_tc2_impl<1, true, 256, 6>(g, tA, tB, ws, dev, dev_err, s, om)
                      : launch_tc2_impl<1, false, 256, 6>(g, tA, tB, ws, dev, dev_err, s, om);
  }
  if (g.dtype == CMPX_F16)
    return g.b_kmajor ? launch_tc2_impl<0, true, 128, 8>(g, tA, tB, ws, dev, dev_err, s, om)
                      : launch_tc2_impl<0, false, 128, 8>(g, tA, tB, ws, dev, dev_err, s, om);
  return g.b_kmajor ? launch_tc2_impl<1, true, 128, 8>(g, tA, tB, ws, dev, dev_err, s, om)
                    : launch_tc2_impl<1, false, 128, 8>(g, tA, tB, ws, dev, dev_err, s, om);
}

}  // namespace cmpx
