// Scaled dot-product attention O = softmax(scale * Q K^T) V for [B, H, S, D]
// tensors, replacing the reference's attention kernels
// (src/cuda/fp16_attention.cu:77 flash_attention_fp16_optimized,
//  src/cuda/bf16_attention.cu:43 attention_bf16_kernel,
//  src/cuda/fp32_attention.cu:35 attention_fp32_strict_kernel;
//  launchers declared at src/main.cpp:48-50, wrapper src/main.cpp:1027-1098).
//
// fp16 / bf16 with D = 64 or 128: tcgen05 flash-attention kernels.  The
// default, attention_pp_kernel (further down), gives each CTA two 128-row
// query tiles so one tile's products run while the other is in softmax.
// The one-tile kernel, attention_tc_kernel: one CTA owns 128 query rows of
// one (batch, head):
//   * warp 0 (TMA): Q once, then K_j and V_j blocks of 128 keys into two
//     separate double-buffered rings (a K slot frees after its QK^T MMA, a V
//     slot after its PV MMA, so the next K block streams in early);
//   * warp 1 (one thread): S_j = Q K_j^T into one of two 128-column TMEM
//     buffers (M 128, N 128, K = D, both operands K-major), then
//     O_j = P_j V_j into one of two D-column TMEM buffers (A = P from shared
//     memory, B = V_j N-major), ordered QK_0, QK_1, PV_0, QK_2, PV_1, ... so
//     one score block is computed while the previous one is in softmax;
//   * warps 2.. (two threads per query row by default, each owning half of
//     the keys of a block and half of the output columns): read S_j from TMEM, keep
//     the running row maximum m (both threads of a row read the whole row,
//     so they agree on it without exchanging anything) and a partial sum l
//     in fp32 (base-2 exponent with scale * log2 e folded in), write their
//     half of P_j = exp2(s - m) as 16-bit values into shared memory in the
//     128-byte-swizzled K-major layout the MMA reads, then fold their half
//     of the previous block's O_{j-1} into fp32 registers:
//     O = O * exp2(m_{j-2} - m_{j-1}) + O_{j-1}.  Finally the two partial
//     sums are combined through shared memory and O / l is rounded once to
//     the output type.
// Every product accumulates in fp32; the reference accumulates fp16 in
// fp16 (src/cuda/fp16_attention.cu:128-239) and normalises with an fp16
// reciprocal, so this kernel's error is an order of magnitude lower.
//
// Other shapes and fp32: a CUDA-core kernel (one warp per query row, the
// same online softmax in fp32, fp32 accumulation).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdio>
#include <cstdlib>

#include "internal.h"
#include "ptx.cuh"

namespace cmpx {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <int D, int TPR>
struct AttnCfg {
  static constexpr int THREADS = 64 + 128 * TPR;     // TMA warp, MMA warp, TPR threads per query row
  static constexpr int SMX = 128 * TPR;              // softmax threads
  static constexpr int QCH = D / 64;                 // 64-element (128-byte) chunks of D
  static constexpr int TILE_BYTES = 128 * D * 2;     // 128 rows x D x 2 B
  static constexpr int P_BYTES = 128 * 128 * 2;      // P block: 128 rows x 128 keys x 2 B
  static constexpr int KST = 2, VST = 2;             // ring depths
  static constexpr size_t SMEM = size_t(TILE_BYTES) * (1 + KST + VST) + 2 * P_BYTES + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = 512;         // S0 S1 (128 each) then O0 O1 (D each)
  static_assert(D == 64 || D == 128, "tensor-core attention supports D = 64 or 128");
  static_assert(TPR == 2 || TPR == 4, "two or four threads per query row");
};

struct AttnParams {
  void* O;
  int S, qtiles;
  float scale_log2;
  int* err;
};

__device__ __forceinline__ void rec_err(int* err, volatile int* abort, int code) {
  *abort = 1;
  atomicCAS(err, 0, code);
}

// 2^x with the hardware's approximate base-2 exponential (ex2.approx,
// relative error ~2^-22; results below 2^-126 flush to zero, which a softmax
// weight that small does not need).  2^-inf = 0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Blackwell's paired fp32 arithmetic: two lanes in one 64-bit register, one
// instruction, each lane rounded exactly as the scalar fmaf / + (.rn), so a
// softmax written with them gives the same bits as the scalar one with about
// half the issue slots.  max3f is the three-input maximum (exact).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// PK = 1: the softmax uses the paired / three-input instructions above (same
// results bit for bit); PK = 0: scalar instructions only.
template <int FMT, int D, int TPR, int PK>
__global__ void __launch_bounds__(AttnCfg<D, TPR>::THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = AttnCfg<D, TPR>;
  using T = typename std::conditional<FMT == 0, __half, __nv_bfloat16>::type;
  constexpr uint32_t IDESC_QK = make_idesc(uint32_t(FMT), 0u, 0u, 128, 128);
  constexpr uint32_t IDESC_PV = make_idesc(uint32_t(FMT), 0u, 1u, 128, D);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::TILE_BYTES;                   // [KST]
  uint8_t* sV = sK + Cfg::KST * Cfg::TILE_BYTES;        // [VST]
  uint8_t* sP = sV + Cfg::VST * Cfg::TILE_BYTES;        // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * Cfg::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + Cfg::KST;
  uint64_t* v_full = k_empty + Cfg::KST;
  uint64_t* v_empty = v_full + Cfg::VST;
  uint64_t* s_full = v_empty + Cfg::VST;   // [2]
  uint64_t* s_empty = s_full + 2;          // [2]
  uint64_t* p_full = s_empty + 2;          // [2]
  uint64_t* o_full = p_full + 2;           // [2]
  uint64_t* o_empty = o_full + 2;          // [2]
  uint64_t* drain = o_empty + 2;
  uint64_t* l_bar = drain + 1;             // the partial row sums are in l_part
  // [TPR][128] partial row sums, written after the last PV MMA has read the
  // P buffers, so they reuse P's space
  float* l_part = reinterpret_cast<float*>(sP);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(l_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / p.qtiles;
  const int q0 = (blockIdx.x - bh * p.qtiles) * 128;
  const int nkv = (p.S + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < Cfg::KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < Cfg::VST; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], Cfg::SMX);
      mbar_init(&p_full[i], Cfg::SMX);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], Cfg::SMX);
    }
    mbar_init(drain, 1);
    mbar_init(l_bar, Cfg::SMX);
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, Cfg::TILE_BYTES);
#pragma unroll
      for (int c = 0; c < Cfg::QCH; ++c) tma_load_3d(sQ + c * 16384, &tmQ, q_full, c * 64, q0, bh);
      bool ok = true;
      int kissued = 0, vissued = 0;
      for (int j = 0; j < nkv && ok; ++j) {
        const int ks = j % Cfg::KST, vs = j % Cfg::VST;
        if (!mbar_wait(&k_empty[ks], ((j / Cfg::KST) & 1) ^ 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutEmpty);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[ks], Cfg::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < Cfg::QCH; ++c)
          tma_load_3d(sK + ks * Cfg::TILE_BYTES + c * 16384, &tmK, &k_full[ks], c * 64, j * 128, bh);
        ++kissued;
        if (!mbar_wait(&v_empty[vs], ((j / Cfg::VST) & 1) ^ 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutEmpty);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[vs], Cfg::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < Cfg::QCH; ++c)
          tma_load_3d(sV + vs * Cfg::TILE_BYTES + c * 16384, &tmV, &v_full[vs], c * 64, j * 128, bh);
        ++vissued;
      }
      if (!ok) {
        // let the copies in flight land before the CTA exits (bounded waits)
        volatile int never = 0;
        mbar_wait(q_full, 0, &never);
        for (int j = (kissued > Cfg::KST ? kissued - Cfg::KST : 0); j < kissued; ++j)
          mbar_wait(&k_full[j % Cfg::KST], (j / Cfg::KST) & 1, &never);
        for (int j = (vissued > Cfg::VST ? vissued - Cfg::VST : 0); j < vissued; ++j)
          mbar_wait(&v_full[j % Cfg::VST], (j / Cfg::VST) & 1, &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag);
      if (!ok) rec_err(p.err, abort_flag, kDevTimeoutFull);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_qk = [&](int j) -> bool {
        const int ks = j % Cfg::KST, b = j & 1;
        if (!mbar_wait(&k_full[ks], (j / Cfg::KST) & 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutFull);
          return false;
        }
        if (!mbar_wait(&s_empty[b], ((j >> 1) & 1) ^ 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutAccEmpty);
          return false;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + ks * Cfg::TILE_BYTES);
        const uint32_t d_tmem = tmem_base + uint32_t(b * 128);
#pragma unroll
        for (int c = 0; c < Cfg::QCH; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(d_tmem, make_sdesc_sw128(q_addr + c * 16384 + kk * 32, 16, 1024),
                    make_sdesc_sw128(k_addr + c * 16384 + kk * 32, 16, 1024), IDESC_QK, (c | kk) != 0 ? 1u : 0u);
        mma_commit(&s_full[b]);
        mma_commit(&k_empty[ks]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int vs = j % Cfg::VST, b = j & 1;
        if (!mbar_wait(&p_full[b], (j >> 1) & 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutFull);
          return false;
        }
        if (!mbar_wait(&v_full[vs], (j / Cfg::VST) & 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutFull);
          return false;
        }
        if (!mbar_wait(&o_empty[b], ((j >> 1) & 1) ^ 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutAccEmpty);
          return false;
        }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + b * Cfg::P_BYTES);
        const uint32_t v_addr = smem_u32(sV + vs * Cfg::TILE_BYTES);
        const uint32_t d_tmem = tmem_base + 256u + uint32_t(b * D);
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(d_tmem, make_sdesc_sw128(p_addr + c2 * 16384 + kk * 32, 16, 1024),
                    make_sdesc_sw128(v_addr + (c2 * 64 + kk * 16) * 128, 16384, 1024), IDESC_PV,
                    (c2 | kk) != 0 ? 1u : 0u);
        mma_commit(&o_full[b]);
        mma_commit(&v_empty[vs]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && nkv > 1) ok = issue_qk(1);
      for (int j = 0; ok && j < nkv; ++j) {
        ok = issue_pv(j);
        if (ok && j + 2 < nkv) ok = issue_qk(j + 2);
      }
      if (!ok) {
        mma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + output (warps 2..)
    constexpr int DH = D / TPR;      // output columns per thread
    constexpr int KPT = 128 / TPR;   // keys of a block per thread
    const int qw = warp & 3;         // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;   // which share of the keys / output columns
    const int r = qw * 32 + lane;    // row of this CTA's 128
    const uint32_t t_lane = tmem_base + (uint32_t(qw * 32) << 16);
    float o[DH];
#pragma unroll
    for (int i = 0; i < DH; ++i) o[i] = 0.0f;
    float m_run = -INFINITY, l = 0.0f;
    float m_prev = -INFINITY;  // running max of the block whose O was folded last
    float m_hist = -INFINITY;  // running max of the block still to fold
    bool ok = true;
    // Iteration j: softmax of block j (j < nkv), then fold O_{j-1} (j >= 1).
    // One fold site keeps the register accumulator in registers.
#pragma unroll 1
    for (int j = 0; j <= nkv; ++j) {
      float m_new = m_run;
      if (j < nkv) {
        const int b = j & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[b], (j >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t s_addr = t_lane + uint32_t(b * 128);
        const int kv0 = j * 128;
        // A block lies wholly inside the keys except possibly the last one.
        const bool full = kv0 + 128 <= p.S;
        const float sl = p.scale_log2;
        // pass 1: the row maximum over all 128 keys of the block, on the raw
        // scores (scaled once at the end; a negative scale needs the minimum,
        // i.e. the maximum of the negated scores).  Eight independent
        // partial maxima per chunk keep the dependent-instruction chains
        // short (a single running maximum is a 128-long serial chain).
        const float sgn = sl >= 0.0f ? 1.0f : -1.0f;
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
        // two halves of 64 scores, each fetched with two loads and one wait
        // (every wait on tensor memory is a full round trip)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t x[64];
          tmem_ld_32x32b_x32(s_addr + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&x[0]));
          tmem_ld_32x32b_x32(s_addr + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&x[32]));
          tmem_ld_wait();
          if (PK && full && sgn > 0.0f) {
#pragma unroll
            for (int i = 0; i < 64; i += 2)
              mx8[(i >> 1) & 7] = max3f(mx8[(i >> 1) & 7], __uint_as_float(x[i]), __uint_as_float(x[i + 1]));
          } else if (PK && full) {
#pragma unroll
            for (int i = 0; i < 64; i += 2)
              mx8[(i >> 1) & 7] = max3f(mx8[(i >> 1) & 7], -__uint_as_float(x[i]), -__uint_as_float(x[i + 1]));
          } else if (full && sgn > 0.0f) {
#pragma unroll
            for (int i = 0; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(x[i]));
          } else if (full) {
#pragma unroll
            for (int i = 0; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], -__uint_as_float(x[i]));
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (kv0 + c * 64 + i < p.S) mx8[i & 7] = fmaxf(mx8[i & 7], sgn * __uint_as_float(x[i]));
          }
        }
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        m_new = fmaxf(m_run, mx * sgn * sl);
        float sum8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sum8[i] = 0.0f;
        // pass 2: this thread's keys [KPT h, KPT (h + 1)): 64-key chunk
        // (KPT h) / 64 of P, 16-byte units from ((KPT h) % 64) / 8 on
        const int key0 = h * KPT;
        uint8_t* prow = sP + b * Cfg::P_BYTES + (key0 >> 6) * 16384 + r * 128;
        const int u0 = (key0 & 63) >> 3;
        uint32_t xk[KPT];  // this thread's scores: all loads issued, then one wait
#pragma unroll
        for (int c = 0; c < KPT / 32; ++c)
          tmem_ld_32x32b_x32(s_addr + key0 + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&xk[c * 32]));
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < KPT / 32; ++c) {
          const uint32_t* x = &xk[c * 32];
          float pv[32];
          if (PK && full) {
            // lanes (i, i + 1) of pair (i & 7) / 2 are sum8[i & 7] and
            // sum8[(i & 7) + 1]: the scalar loop's association exactly
            const uint64_t sl2 = f2pack(sl, sl), nm2 = f2pack(-m_new, -m_new);
            uint64_t s2[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) s2[k] = f2pack(sum8[2 * k], sum8[2 * k + 1]);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float2 t = f2unpack(fma2(f2pack(__uint_as_float(x[i]), __uint_as_float(x[i + 1])), sl2, nm2));
              pv[i] = ex2_approx(t.x);
              pv[i + 1] = ex2_approx(t.y);
              s2[(i & 7) >> 1] = add2(s2[(i & 7) >> 1], f2pack(pv[i], pv[i + 1]));
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 t = f2unpack(s2[k]);
              sum8[2 * k] = t.x;
              sum8[2 * k + 1] = t.y;
            }
          } else if (full) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              pv[i] = ex2_approx(fmaf(__uint_as_float(x[i]), sl, -m_new));
              sum8[i & 7] += pv[i];
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              pv[i] = (kv0 + key0 + c * 32 + i < p.S) ? ex2_approx(fmaf(__uint_as_float(x[i]), sl, -m_new)) : 0.0f;
              sum8[i & 7] += pv[i];
            }
          }
          // 16-byte unit u of the row's 128 bytes holds keys [8u, 8u + 8) of the chunk
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 q;
            q.x = pack2(pv[g * 8 + 0], pv[g * 8 + 1], (T*)nullptr);
            q.y = pack2(pv[g * 8 + 2], pv[g * 8 + 3], (T*)nullptr);
            q.z = pack2(pv[g * 8 + 4], pv[g * 8 + 5], (T*)nullptr);
            q.w = pack2(pv[g * 8 + 6], pv[g * 8 + 7], (T*)nullptr);
            const int u = u0 + c * 4 + g;
            *reinterpret_cast<uint4*>(prow + ((u ^ (r & 7)) << 4)) = q;
          }
        }
        const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
        l = l * ex2_approx(m_run - m_new) + sum;
        m_run = m_new;
        tc_fence_before();
        mbar_arrive(&s_empty[b]);   // S buffer may be overwritten by QK_{j+2}
        fence_proxy_async_smem();   // P visible to the tensor core
        mbar_arrive(&p_full[b]);
      }
      if (j >= 1) {
        const int b = (j - 1) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&o_full[b], ((j - 1) >> 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float beta = ex2_approx(m_prev - m_hist);  // 0 while nothing has been folded
        // this thread's DH columns of O_{j-1}: all loads issued, then one wait
        {
          uint32_t x[DH];
#pragma unroll
          for (int c = 0; c < DH / 16; ++c)
            tmem_ld_32x32b_x16(t_lane + 256u + uint32_t(b * D + h * DH + c * 16),
                               *reinterpret_cast<uint32_t(*)[16]>(&x[c * 16]));
          tmem_ld_wait();
          if (PK) {
            const uint64_t b2 = f2pack(beta, beta);
#pragma unroll
            for (int i = 0; i < DH; i += 2) {
              const float2 t = f2unpack(
                  fma2(f2pack(o[i], o[i + 1]), b2, f2pack(__uint_as_float(x[i]), __uint_as_float(x[i + 1]))));
              o[i] = t.x;
              o[i + 1] = t.y;
            }
          } else {
#pragma unroll
            for (int i = 0; i < DH; ++i) o[i] = fmaf(o[i], beta, __uint_as_float(x[i]));
          }
        }
        tc_fence_before();
        mbar_arrive(&o_empty[b]);
        m_prev = m_hist;
      }
      m_hist = m_new;
    }
    if (ok) {
      // combine the two partial row sums (bounded wait: a thread that gave
      // up never arrives, and its partner then gives up too)
      l_part[h * 128 + r] = l;
      mbar_arrive(l_bar);
      ok = __all_sync(0xffffffffu, mbar_wait(l_bar, 0, abort_flag));
    }
    if (!ok) {
      if (lane == 0) rec_err(p.err, abort_flag, kDevTimeoutAccFull);
    } else if (q0 + r < p.S) {
      float lsum = 0.0f;
#pragma unroll
      for (int t = 0; t < TPR; ++t) lsum += l_part[t * 128 + r];
      const float inv = 1.0f / lsum;
      T* orow = reinterpret_cast<T*>(p.O) + (size_t(bh) * p.S + q0 + r) * D + h * DH;
#pragma unroll
      for (int g = 0; g < DH / 8; ++g) {
        uint4 q;
        q.x = pack2(o[g * 8 + 0] * inv, o[g * 8 + 1] * inv, (T*)nullptr);
        q.y = pack2(o[g * 8 + 2] * inv, o[g * 8 + 3] * inv, (T*)nullptr);
        q.z = pack2(o[g * 8 + 4] * inv, o[g * 8 + 5] * inv, (T*)nullptr);
        q.w = pack2(o[g * 8 + 6] * inv, o[g * 8 + 7] * inv, (T*)nullptr);
        reinterpret_cast<uint4*>(orow)[g] = q;
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

// ------------------------------------------------- two query tiles per CTA
// attention_pp_kernel: one CTA owns 256 query rows (tiles A and B) of one
// (batch, head), so the tensor core works on one tile's products while the
// other tile is in softmax:
//   * warp 0 (TMA): both Q tiles once, then K_0, V_0, K_1, V_1, ... into
//     a K ring and a V ring;
//   * warp 1 (one thread): S_t = Q_t K_j^T into tile t's 128-column TMEM
//     buffer as soon as tile t's softmax has read the previous S_t out and
//     K_j is in, and O_t += P_t V_j into tile t's D-column accumulator once
//     P_t is written and V_j is in, for both tiles in whichever order their
//     inputs become ready;
//   * warps 2-5 (tile A) and 6-9 (tile B): one thread per query row, holding
//     the row's 128 scores of a block in registers: the running maximum and
//     sum in fp32, P = exp2(s * scale * log2 e - m) as 16-bit values into
//     shared memory (128-byte-swizzled K-major), and, when a row's maximum
//     grew, O_t in tensor memory scaled by exp2(m_old - m_new) before the
//     next P_t V_j accumulates into it (the factor is exactly 1 when the
//     maximum did not move, so skipping that case changes nothing).  At the
//     end O_t / l is rounded once.
template <int D>
struct PPCfg {
  static constexpr int THREADS = 64 + 256;         // TMA warp, MMA warp, 2 x 4 softmax warps
  static constexpr int QCH = D / 64;
  static constexpr int TILE_BYTES = 128 * D * 2;
  static constexpr int P_BYTES = 128 * 128 * 2;
  // K_j in slot j % KS, V_j in slot KS + j % VS.  With one K slot, K_{j+1}
  // loads as soon as the last Q K_j^T is done; two V slots let V_{j+1} load a
  // whole block ahead of its first P V.
  static constexpr int KS = D == 128 ? 1 : 3;
  static constexpr int VS = D == 128 ? 2 : 3;
  static constexpr int NS = KS + VS;               // K/V slots
  static constexpr size_t SMEM = size_t(TILE_BYTES) * (2 + NS) + 2 * P_BYTES + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = 512;       // S_A S_B (128 each), O_A O_B (D each)
  static_assert(D == 64 || D == 128, "tensor-core attention supports D = 64 or 128");
};

template <int FMT, int D>
__global__ void __launch_bounds__(PPCfg<D>::THREADS, 1)
    attention_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using Cfg = PPCfg<D>;
  using T = typename std::conditional<FMT == 0, __half, __nv_bfloat16>::type;
  constexpr int NS = Cfg::NS;
  constexpr uint32_t IDESC_QK = make_idesc(uint32_t(FMT), 0u, 0u, 128, 128);
  constexpr uint32_t IDESC_PV = make_idesc(uint32_t(FMT), 0u, 1u, 128, D);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
  uint8_t* sQ = smem;                                  // [2] tiles
  uint8_t* sKV = sQ + 2 * Cfg::TILE_BYTES;             // [NS] slots
  uint8_t* sP = sKV + NS * Cfg::TILE_BYTES;            // [2] tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * Cfg::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;        // [NS]
  uint64_t* kv_empty = kv_full + NS;     // [NS]
  uint64_t* s_full = kv_empty + NS;      // [2] S_t computed
  uint64_t* s_free = s_full + 2;         // [2] S_t read out by tile t's softmax
  uint64_t* p_full = s_free + 2;         // [2] P_t written and O_t rescaled
  uint64_t* o_full = p_full + 2;         // [2] P_t V_j accumulated into O_t
  uint64_t* drain = o_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / p.qtiles;                 // qtiles = CTAs per (batch, head) here
  const int q0 = (blockIdx.x - bh * p.qtiles) * 256;
  const int nt = q0 + 128 < p.S ? 2 : 1;                // query tiles of this CTA
  const int nkv = (p.S + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(q_full, uint32_t(nt * Cfg::TILE_BYTES));
      for (int t = 0; t < nt; ++t)
#pragma unroll
        for (int c = 0; c < Cfg::QCH; ++c)
          tma_load_3d(sQ + t * Cfg::TILE_BYTES + c * 16384, &tmQ, q_full, c * 64, q0 + t * 128, bh);
      // K_0, V_0, K_1, V_1, ... each into its own ring
      int issued[NS];
#pragma unroll
      for (int i = 0; i < NS; ++i) issued[i] = 0;
      bool ok = true;
      for (int i = 0; i < 2 * nkv && ok; ++i) {
        const int j = i >> 1;
        const bool isv = (i & 1) != 0;
        const int slot = isv ? Cfg::KS + j % Cfg::VS : j % Cfg::KS;
        const int use = isv ? j / Cfg::VS : j / Cfg::KS;   // earlier loads into this slot
        if (!mbar_wait(&kv_empty[slot], (use & 1) ^ 1, abort_flag)) {
          rec_err(p.err, abort_flag, kDevTimeoutEmpty);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[slot], Cfg::TILE_BYTES);
        const CUtensorMap* m = isv ? &tmV : &tmK;
#pragma unroll
        for (int c = 0; c < Cfg::QCH; ++c)
          tma_load_3d(sKV + slot * Cfg::TILE_BYTES + c * 16384, m, &kv_full[slot], c * 64, j * 128, bh);
        issued[slot] = use + 1;
      }
      if (!ok) {
        // let the copies in flight land before the CTA exits (bounded waits;
        // a slot's loads complete in order, so its last one is enough)
        volatile int never = 0;
        mbar_wait(q_full, 0, &never);
        for (int i = 0; i < NS; ++i)
          if (issued[i] > 0) mbar_wait(&kv_full[i], (issued[i] - 1) & 1, &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag);
      if (!ok) rec_err(p.err, abort_flag, kDevTimeoutFull);
      auto k_ready = [&](int j) { return mbar_try_wait(&kv_full[j % Cfg::KS], (j / Cfg::KS) & 1); };
      auto v_ready = [&](int j) { return mbar_try_wait(&kv_full[Cfg::KS + j % Cfg::VS], (j / Cfg::VS) & 1); };
      auto qk = [&](int t, int j) {
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + t * Cfg::TILE_BYTES);
        const uint32_t k_addr = smem_u32(sKV + (j % Cfg::KS) * Cfg::TILE_BYTES);
        const uint32_t d_tmem = tmem_base + uint32_t(t * 128);
#pragma unroll
        for (int c = 0; c < Cfg::QCH; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(d_tmem, make_sdesc_sw128(q_addr + c * 16384 + kk * 32, 16, 1024),
                    make_sdesc_sw128(k_addr + c * 16384 + kk * 32, 16, 1024), IDESC_QK, (c | kk) != 0 ? 1u : 0u);
        mma_commit(&s_full[t]);
      };
      auto pv = [&](int t, int j) {
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + t * Cfg::P_BYTES);
        const uint32_t v_addr = smem_u32(sKV + (Cfg::KS + j % Cfg::VS) * Cfg::TILE_BYTES);
        const uint32_t d_tmem = tmem_base + 256u + uint32_t(t * D);
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16(d_tmem, make_sdesc_sw128(p_addr + c2 * 16384 + kk * 32, 16, 1024),
                    make_sdesc_sw128(v_addr + (c2 * 64 + kk * 16) * 128, 16384, 1024), IDESC_PV,
                    (j | c2 | kk) != 0 ? 1u : 0u);
        mma_commit(&o_full[t]);
      };
      if (ok) {
        ok = mbar_wait(&kv_full[0], 0, abort_flag);
        if (!ok) rec_err(p.err, abort_flag, kDevTimeoutFull);
      }
      if (ok) {
        for (int t = 0; t < nt; ++t) qk(t, 0);
        mma_commit(&kv_empty[0]);
      }
      // Per block j, for both tiles t: S_t = Q_t K_{j+1}^T (needs K_{j+1}
      // and S_t read out) and O_t += P_t V_j (needs P_t and V_j), each issued
      // as soon as its inputs are ready (bounded polling), so a late tile
      // does not hold up the other.
      for (int j = 0; ok && j < nkv; ++j) {
        const bool more = j + 1 < nkv;
        bool need_qk[2] = {more, more && nt > 1};
        bool need_pv[2] = {true, nt > 1};
        bool k_in = false, v_in = false;
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t it = 1; need_qk[0] || need_qk[1] || need_pv[0] || need_pv[1]; ++it) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (need_qk[t] && (k_in || (k_in = k_ready(j + 1))) && mbar_try_wait(&s_free[t], j & 1)) {
              qk(t, j + 1);
              need_qk[t] = false;
              if (!need_qk[0] && !need_qk[1]) mma_commit(&kv_empty[(j + 1) % Cfg::KS]);
            }
            if (need_pv[t] && (v_in || (v_in = v_ready(j))) && mbar_try_wait(&p_full[t], j & 1)) {
              pv(t, j);
              need_pv[t] = false;
            }
          }
          if ((it & 63u) == 0 && (*abort_flag || globaltimer_ns() - t0 > CMPX_WAIT_TIMEOUT_NS)) {
            rec_err(p.err, abort_flag, kDevTimeoutFull);
            ok = false;
            break;
          }
        }
        if (ok) mma_commit(&kv_empty[Cfg::KS + j % Cfg::VS]);
      }
      if (!ok) {
        mma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never);
      }
    }
  } else if ((warp - 2) >> 2 < nt) {
    // ------------------------------------------------------------ softmax + output (warps 2..9)
    const int t = (warp - 2) >> 2;   // query tile
    const int qw = warp & 3;         // TMEM lane quarter this warp may access
    const int r = qw * 32 + lane;    // row of the tile
    const uint32_t t_lane = tmem_base + (uint32_t(qw * 32) << 16);
    const uint32_t s_col = uint32_t(t * 128), o_col = 256u + uint32_t(t * D);
    const float sl = p.scale_log2;
    const float sgn = sl >= 0.0f ? 1.0f : -1.0f;
    uint8_t* prow = sP + t * Cfg::P_BYTES + r * 128;
    float m_run = -INFINITY, l = 0.0f;
    bool ok = true;
#pragma unroll 1
    for (int j = 0; j < nkv; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t x[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld_32x32b_x32(t_lane + s_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&x[c * 32]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_free[t]);   // S_t may be overwritten by the next block's QK
      const int kv0 = j * 128;
      const bool full = kv0 + 128 <= p.S;
      // the row maximum on the raw scores (of the negated ones for a negative
      // scale), four independent partial maxima (eight, or eight partial sums
      // below, and the compiler spills at the 168-register cap)
      float mx4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) mx4[i] = -INFINITY;
      if (full && sgn > 0.0f) {
#pragma unroll
        for (int i = 0; i < 128; i += 2)
          mx4[(i >> 1) & 3] = max3f(mx4[(i >> 1) & 3], __uint_as_float(x[i]), __uint_as_float(x[i + 1]));
      } else if (full) {
#pragma unroll
        for (int i = 0; i < 128; i += 2)
          mx4[(i >> 1) & 3] = max3f(mx4[(i >> 1) & 3], -__uint_as_float(x[i]), -__uint_as_float(x[i + 1]));
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kv0 + i < p.S) mx4[i & 3] = fmaxf(mx4[i & 3], sgn * __uint_as_float(x[i]));
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      const float m_new = fmaxf(m_run, mx * sgn * sl);
      const float alpha = ex2_approx(m_run - m_new);   // 0 for the first block, 1 when m did not move
      // P = exp2(s * sl - m_new) in place of the scores, with the row sum
      uint64_t s2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) s2[k] = f2pack(0.0f, 0.0f);
      const uint64_t sl2 = f2pack(sl, sl), nm2 = f2pack(-m_new, -m_new);
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        const float2 a = f2unpack(fma2(f2pack(__uint_as_float(x[i]), __uint_as_float(x[i + 1])), sl2, nm2));
        float e0 = ex2_approx(a.x), e1 = ex2_approx(a.y);
        if (!full) {
          if (kv0 + i >= p.S) e0 = 0.0f;
          if (kv0 + i + 1 >= p.S) e1 = 0.0f;
        }
        x[i] = __float_as_uint(e0);
        x[i + 1] = __float_as_uint(e1);
        s2[(i >> 1) & 1] = add2(s2[(i >> 1) & 1], f2pack(e0, e1));
      }
      float sum = 0.0f;
      {
        const float2 a = f2unpack(s2[0]), b = f2unpack(s2[1]);
        sum = (a.x + a.y) + (b.x + b.y);
      }
      l = l * alpha + sum;
      if (j >= 1) {
        // P_t V_{j-1} done: P_t's buffer is free and O_t holds the sum so far
        if (!__all_sync(0xffffffffu, mbar_wait(&o_full[t], (j - 1) & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // 16-byte unit u of a 64-key chunk's 128-byte row holds keys [8u, 8u + 8)
#pragma unroll
      for (int g = 0; g < 16; ++g) {
        uint4 q;
        q.x = pack2(__uint_as_float(x[g * 8 + 0]), __uint_as_float(x[g * 8 + 1]), (T*)nullptr);
        q.y = pack2(__uint_as_float(x[g * 8 + 2]), __uint_as_float(x[g * 8 + 3]), (T*)nullptr);
        q.z = pack2(__uint_as_float(x[g * 8 + 4]), __uint_as_float(x[g * 8 + 5]), (T*)nullptr);
        q.w = pack2(__uint_as_float(x[g * 8 + 6]), __uint_as_float(x[g * 8 + 7]), (T*)nullptr);
        const int u = g & 7;
        *reinterpret_cast<uint4*>(prow + (g >> 3) * 16384 + ((u ^ (r & 7)) << 4)) = q;
      }
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // the whole D-column row of O_t in one load round trip (the score
        // registers are free again once P is stored)
        const uint64_t a2 = f2pack(alpha, alpha);
        uint32_t y[D];
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tmem_ld_32x32b_x32(t_lane + o_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&y[c * 32]));
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < D; i += 2) {
          const float2 v = f2unpack(mul2(f2pack(__uint_as_float(y[i]), __uint_as_float(y[i + 1])), a2));
          y[i] = __float_as_uint(v.x);
          y[i + 1] = __float_as_uint(v.y);
        }
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tmem_st_32x32b_x32(t_lane + o_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&y[c * 32]));
        tmem_st_wait();
      }
      tc_fence_before();
      fence_proxy_async_smem();   // P visible to the tensor core
      mbar_arrive(&p_full[t]);
      m_run = m_new;
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&o_full[t], (nkv - 1) & 1, abort_flag));
    if (!ok) {
      if (lane == 0) rec_err(p.err, abort_flag, kDevTimeoutAccFull);
    } else {
      tc_fence_after();
      const float inv = 1.0f / l;
      const int row = q0 + t * 128 + r;
      T* orow = reinterpret_cast<T*>(p.O) + (size_t(bh) * p.S + row) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t y[32];
        tmem_ld_32x32b_x32(t_lane + o_col + c * 32, y);
        tmem_ld_wait();
        if (row < p.S) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 q;
            q.x = pack2(__uint_as_float(y[g * 8 + 0]) * inv, __uint_as_float(y[g * 8 + 1]) * inv, (T*)nullptr);
            q.y = pack2(__uint_as_float(y[g * 8 + 2]) * inv, __uint_as_float(y[g * 8 + 3]) * inv, (T*)nullptr);
            q.z = pack2(__uint_as_float(y[g * 8 + 4]) * inv, __uint_as_float(y[g * 8 + 5]) * inv, (T*)nullptr);
            q.w = pack2(__uint_as_float(y[g * 8 + 6]) * inv, __uint_as_float(y[g * 8 + 7]) * inv, (T*)nullptr);
            reinterpret_cast<uint4*>(orow + c * 32)[g] = q;
          }
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

// ------------------------------------------------------------------ CUDA cores
template <typename T>
__device__ __forceinline__ float ldf(const T* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__half* p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ void stf(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// One warp per query row; lane d holds output columns d, d+32, ... (up to
// kSimtMaxD / 32 of them).  Online softmax in fp32 over all S keys.
constexpr int kSimtMaxD = 512;

template <typename T>
__global__ void __launch_bounds__(128) attention_simt_kernel(const T* __restrict__ Q, const T* __restrict__ K,
                                                             const T* __restrict__ V, T* __restrict__ O,
                                                             long long rows, int S, int D, float scale_log2) {
  const long long row = blockIdx.x * 4LL + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long bh = row / S;
  const T* q = Q + row * D;
  const T* kb = K + bh * S * (long long)D;
  const T* vb = V + bh * S * (long long)D;
  constexpr int NV = kSimtMaxD / 32;
  float qv[NV], acc[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < D ? ldf(q + d) : 0.0f;
    acc[i] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  for (int k = 0; k < S; ++k) {
    const T* kr = kb + (long long)k * D;
    float dot = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int d = lane + 32 * i;
      if (d < D) dot = fmaf(qv[i], ldf(kr + d), dot);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float s = dot * scale_log2;
    const float m_new = fmaxf(m, s);
    const float alpha = exp2f(m - m_new);
    const float pk = exp2f(s - m_new);
    l = l * alpha + pk;
    const T* vr = vb + (long long)k * D;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int d = lane + 32 * i;
      if (d < D) acc[i] = fmaf(acc[i], alpha, pk * ldf(vr + d));
    }
    m = m_new;
  }
  const float inv = 1.0f / l;
  T* orow = O + row * D;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int d = lane + 32 * i;
    if (d < D) stf(orow + d, acc[i] * inv);
  }
}

template <int FMT, int D, int TPR, int PK>
cudaError_t launch_tc(const void* Q, const void* K, const void* V, void* O, int64_t BH, int64_t S, float scale,
                      int* err, cudaStream_t s) {
  using Cfg = AttnCfg<D, TPR>;
  auto kern = attention_tc_kernel<FMT, D, TPR, PK>;
  static_assert(Cfg::SMEM <= 232448, "shared memory budget");
  static unsigned long long smem_set = 0;
  cudaError_t e = set_smem_once(kern, int(Cfg::SMEM), smem_set);
  if (e != cudaSuccess) return e;
  const int dt = FMT == 0 ? CMPX_F16 : CMPX_BF16;
  CUtensorMap tq, tk, tv;
  if (encode_tmap_3d(&tq, dt, Q, D, S, BH, D, S * D, 64, 128) != CMPX_OK ||
      encode_tmap_3d(&tk, dt, K, D, S, BH, D, S * D, 64, 128) != CMPX_OK ||
      encode_tmap_3d(&tv, dt, V, D, S, BH, D, S * D, 64, 128) != CMPX_OK)
    return cudaErrorInvalidValue;
  AttnParams p;
  p.O = O;
  p.S = int(S);
  p.qtiles = int((S + 127) / 128);
  p.scale_log2 = scale * kLog2e;
  p.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(BH * p.qtiles));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  apply_pdl(cfg, attr, 0);
  return cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, p);
}

template <int FMT, int D>
cudaError_t launch_pp(const void* Q, const void* K, const void* V, void* O, int64_t BH, int64_t S, float scale,
                      int* err, cudaStream_t s) {
  using Cfg = PPCfg<D>;
  auto kern = attention_pp_kernel<FMT, D>;
  static_assert(Cfg::SMEM <= 232448, "shared memory budget");
  static unsigned long long smem_set = 0;
  cudaError_t e = set_smem_once(kern, int(Cfg::SMEM), smem_set);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "cmpx attention (two-tile kernel) shared memory %zu: %s\n", size_t(Cfg::SMEM),
                 cudaGetErrorString(e));
    return e;
  }
  const int dt = FMT == 0 ? CMPX_F16 : CMPX_BF16;
  CUtensorMap tq, tk, tv;
  if (encode_tmap_3d(&tq, dt, Q, D, S, BH, D, S * D, 64, 128) != CMPX_OK ||
      encode_tmap_3d(&tk, dt, K, D, S, BH, D, S * D, 64, 128) != CMPX_OK ||
      encode_tmap_3d(&tv, dt, V, D, S, BH, D, S * D, 64, 128) != CMPX_OK)
    return cudaErrorInvalidValue;
  AttnParams p;
  p.O = O;
  p.S = int(S);
  p.qtiles = int(((S + 127) / 128 + 1) / 2);   // CTAs (pairs of 128-row tiles) per (batch, head)
  p.scale_log2 = scale * kLog2e;
  p.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(BH * p.qtiles));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  apply_pdl(cfg, attr, 0);
  e = cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, p);
  if (e != cudaSuccess) {
    cudaFuncAttributes fa = {};
    cudaFuncGetAttributes(&fa, kern);
    std::fprintf(stderr, "cmpx attention (two-tile kernel) launch: %s (registers %d, max threads %d, smem %zu)\n",
                 cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, size_t(Cfg::SMEM));
  }
  return e;
}

template <typename T>
cudaError_t launch_simt_attn(const void* Q, const void* K, const void* V, void* O, int64_t BH, int64_t S, int64_t D,
                             float scale, cudaStream_t s) {
  const long long rows = BH * S;
  const long long blocks = (rows + 3) / 4;
  attention_simt_kernel<T><<<unsigned(blocks), 128, 0, s>>>(static_cast<const T*>(Q), static_cast<const T*>(K),
                                                            static_cast<const T*>(V), static_cast<T*>(O), rows,
                                                            int(S), int(D), scale * kLog2e);
  return cudaGetLastError();
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Softmax threads per query row of the tensor-core kernel: 2 by default,
// 4 with CMPX_ATTN_TPR=4 (twice the warps to hide latency, but every thread
// still reads the whole score row for the maximum; measured on a B200 on
// 8x8x1024x128 fp16: 503 TFLOP/s with 2, 477 with 4).
int attention_threads_per_row() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("CMPX_ATTN_TPR");
    v = (e != nullptr && e[0] == '4') ? 4 : 2;
  }
  return v;
}

// The softmax of the two-threads-per-row kernel in paired fp32 / three-input
// max instructions (default), or in scalar ones with CMPX_ATTN_PACKED=0; the
// results are the same bit for bit.
// The tensor-core kernel: two query tiles per CTA (attention_pp_kernel) by
// default; the one-tile kernel (attention_tc_kernel) with CMPX_ATTN_KERNEL=one
// (measured on a B200, 8x8x1024x128 fp16: 624-626 vs 544-546 TFLOP/s).
bool attention_pingpong() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("CMPX_ATTN_KERNEL");
    v = (e != nullptr && e[0] == 'o') ? 0 : 1;
  }
  return v == 1;
}

bool attention_packed() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("CMPX_ATTN_PACKED");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

}  // namespace

int attention_path(int dtype, const void* Q, const void* K, const void* V, const void* O, int64_t D, int requested) {
  const bool tc_ok = (dtype == CMPX_F16 || dtype == CMPX_BF16) && (D == 64 || D == 128) && al16(Q) && al16(K) &&
                     al16(V) && al16(O);
  if (requested == CMPX_PATH_TC) return tc_ok ? CMPX_PATH_TC : -1;
  if (requested == CMPX_PATH_SIMT) return D <= kSimtMaxD ? CMPX_PATH_SIMT : -1;
  if (requested != CMPX_PATH_AUTO) return -1;
  if (tc_ok) return CMPX_PATH_TC;
  return D <= kSimtMaxD ? CMPX_PATH_SIMT : -1;
}

}  // namespace cmpx

using namespace cmpx;

extern "C" int cmpx_attention(int dtype, const void* Q, const void* K, const void* V, void* O, int64_t B, int64_t H,
                              int64_t S, int64_t D, float scale, int path, cmpx_stream_t stream) {
  if (dtype != CMPX_F16 && dtype != CMPX_BF16 && dtype != CMPX_F32) return CMPX_ERR_INVALID_ARG;
  if (B < 0 || H < 0 || S < 0 || D < 0) return CMPX_ERR_INVALID_ARG;
  if (B == 0 || H == 0 || S == 0 || D == 0) return CMPX_OK;
  if (Q == nullptr || K == nullptr || V == nullptr || O == nullptr) return CMPX_ERR_INVALID_ARG;
  if (S > (int64_t(1) << 31) - 1 || B * H > (int64_t(1) << 31) - 1) return CMPX_ERR_UNSUPPORTED;
  const int pth = attention_path(dtype, Q, K, V, O, D, path);
  if (pth < 0) return CMPX_ERR_UNSUPPORTED;
  DeviceInfo dev;
  int* err = nullptr;
  int st = device_facts(&dev, &err);
  if (st != CMPX_OK) return st;
  const int64_t BH = B * H;
  cudaError_t e;
  if (pth == CMPX_PATH_TC) {
    if (BH * ((S + 127) / 128) > 0x7fffffffLL) return CMPX_ERR_UNSUPPORTED;
    const bool four = attention_threads_per_row() == 4;
    const bool packed = attention_packed();
    if (attention_pingpong()) {
      if (dtype == CMPX_F16)
        e = D == 64 ? launch_pp<0, 64>(Q, K, V, O, BH, S, scale, err, stream)
                    : launch_pp<0, 128>(Q, K, V, O, BH, S, scale, err, stream);
      else
        e = D == 64 ? launch_pp<1, 64>(Q, K, V, O, BH, S, scale, err, stream)
                    : launch_pp<1, 128>(Q, K, V, O, BH, S, scale, err, stream);
    } else if (dtype == CMPX_F16) {
      if (D == 64)
        e = four ? launch_tc<0, 64, 4, 0>(Q, K, V, O, BH, S, scale, err, stream)
             : packed ? launch_tc<0, 64, 2, 1>(Q, K, V, O, BH, S, scale, err, stream)
                      : launch_tc<0, 64, 2, 0>(Q, K, V, O, BH, S, scale, err, stream);
      else
        e = four ? launch_tc<0, 128, 4, 0>(Q, K, V, O, BH, S, scale, err, stream)
             : packed ? launch_tc<0, 128, 2, 1>(Q, K, V, O, BH, S, scale, err, stream)
                      : launch_tc<0, 128, 2, 0>(Q, K, V, O, BH, S, scale, err, stream);
    } else {
      if (D == 64)
        e = four ? launch_tc<1, 64, 4, 0>(Q, K, V, O, BH, S, scale, err, stream)
             : packed ? launch_tc<1, 64, 2, 1>(Q, K, V, O, BH, S, scale, err, stream)
                      : launch_tc<1, 64, 2, 0>(Q, K, V, O, BH, S, scale, err, stream);
      else
        e = four ? launch_tc<1, 128, 4, 0>(Q, K, V, O, BH, S, scale, err, stream)
             : packed ? launch_tc<1, 128, 2, 1>(Q, K, V, O, BH, S, scale, err, stream)
                      : launch_tc<1, 128, 2, 0>(Q, K, V, O, BH, S, scale, err, stream);
    }
  } else {
    if ((BH * S + 3) / 4 > 0x7fffffffLL) return CMPX_ERR_UNSUPPORTED;
    e = dtype == CMPX_F16    ? launch_simt_attn<__half>(Q, K, V, O, BH, S, D, scale, stream)
        : dtype == CMPX_BF16 ? launch_simt_attn<__nv_bfloat16>(Q, K, V, O, BH, S, D, scale, stream)
                             : launch_simt_attn<float>(Q, K, V, O, BH, S, D, scale, stream);
  }
  return e == cudaSuccess ? CMPX_OK : CMPX_ERR_CUDA;
}

extern "C" int cmpx_attention_select_path(int dtype, const void* Q, const void* K, const void* V, const void* O,
                                          int64_t D, int path) {
  if (dtype != CMPX_F16 && dtype != CMPX_BF16 && dtype != CMPX_F32) return -1;
  return attention_path(dtype, Q, K, V, O, D, path);
}

// Reference-compatible C++-linkage launchers (src/main.cpp:48-50): legacy
// default stream, no status; a failure is reported on stderr.
static void report_attn(const char* what, int st) {
  if (st != CMPX_OK) fprintf(stderr, "cmpx %s error: %s\n", what, cmpx_status_string(st));
}
CMPX_API void launch_attention_fp32(const float* q, const float* k, const float* v, float* output, int B, int H, int S,
                                    int D, float scale) {
  report_attn("launch_attention_fp32", cmpx_attention(CMPX_F32, q, k, v, output, B, H, S, D, scale, 0, nullptr));
}
CMPX_API void launch_attention_fp16(const void* q, const void* k, const void* v, void* output, int B, int H, int S,
                                    int D, float scale) {
  report_attn("launch_attention_fp16", cmpx_attention(CMPX_F16, q, k, v, output, B, H, S, D, scale, 0, nullptr));
}
CMPX_API void launch_attention_bf16(const void* q, const void* k, const void* v, void* output, int B, int H, int S,
                                    int D, float scale) {
  report_attn("launch_attention_bf16", cmpx_attention(CMPX_BF16, q, k, v, output, B, H, S, D, scale, 0, nullptr));
}
