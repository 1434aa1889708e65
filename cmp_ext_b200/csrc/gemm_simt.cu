// CUDA-core fallback GEMM, bias add and K == 0 fill.
//
// The fallback covers what the TMA paths cannot describe: row strides that
// are not a multiple of 16 bytes (e.g. the reference's fp32 odd-shape case,
// K = 511), unaligned base pointers, and tiny problems.  Like the reference's
// gemm_fp32_ga100_kernel (src/cuda/fp32_matmul.cu:31-184) it handles any
// M, N, K with bounds checks; unlike it, it accumulates in fp32 with FMA for
// every dtype (the reference accumulates fp16/bf16 in half precision,
// src/cuda/fp16_matmul.cu:225-226, src/cuda/bf16_matmul.cu:196).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace cmpx {
namespace {

__device__ __forceinline__ float ld_f32(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float ld_f32(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float ld_f32(const float* p) { return *p; }
__device__ __forceinline__ void st_f32(__half* p, float v) { *p = __float2half_rn(v); }
__device__ __forceinline__ void st_f32(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void st_f32(float* p, float v) { *p = v; }

constexpr int SB_M = 128, SB_N = 128, SB_K = 8, SB_PAD = 4;

// 256 threads, each computes an 8x8 block of a 128x128 tile: rows
// {ty*4 .. ty*4+3, 64+ty*4 .. 64+ty*4+3}, columns likewise from tx, so the
// operands come out of shared memory as float4s with few bank conflicts.
// K advances 8 at a time through a double-buffered shared-memory tile; the
// next tile's global loads are held in registers while the current one is
// multiplied.  Every global access is bounds-checked and uses the caller's
// strides (any alignment).  blockIdx.z = batch.
template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                        T* __restrict__ C, const T* __restrict__ bias, int M, int N,
                                                        int K, long long lda, long long ldb, long long ldc,
                                                        long long sa, long long sb, long long sc, int b_kmajor,
                                                        int bias_m, PeerOut peers) {
  __shared__ __align__(16) float As[2][SB_K][SB_M + SB_PAD];
  __shared__ __align__(16) float Bs[2][SB_K][SB_N + SB_PAD];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * SB_M, n0 = blockIdx.x * SB_N;
  const long long bz = blockIdx.z;
  A += bz * sa;
  B += bz * sb;
  C += bz * sc;
  // global -> register staging: 4 A values (row tid/2, k (tid%2)*4 + 0..3)
  // and 4 B values (B [K,N]: k tid/32, columns (tid%32)*4 + 0..3;
  // B [N,K]: column tid/2, k (tid%2)*4 + 0..3)
  float ra[4], rb[4];
  const int a_r = tid >> 1, a_k = (tid & 1) * 4;
  auto load = [&](int k0) {
    const int gm = m0 + a_r;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gk = k0 + a_k + i;
      ra[i] = (gm < M && gk < K) ? ld_f32(A + gm * lda + gk) : 0.0f;
    }
    if (b_kmajor) {
      const int gn = n0 + a_r;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int gk = k0 + a_k + i;
        rb[i] = (gn < N && gk < K) ? ld_f32(B + gn * ldb + gk) : 0.0f;
      }
    } else {
      const int gk = k0 + (tid >> 5);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int gn = n0 + (tid & 31) * 4 + i;
        rb[i] = (gn < N && gk < K) ? ld_f32(B + gk * ldb + gn) : 0.0f;
      }
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) As[buf][a_k + i][a_r] = ra[i];
    if (b_kmajor) {
#pragma unroll
      for (int i = 0; i < 4; ++i) Bs[buf][a_k + i][a_r] = rb[i];
    } else {
      *reinterpret_cast<float4*>(&Bs[buf][tid >> 5][(tid & 31) * 4]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
    }
  };
  float acc[8][8] = {};
  const int nk = (K + SB_K - 1) / SB_K;
  load(0);
  store(0);
  __syncthreads();
  for (int t = 0; t < nk; ++t) {
    const int buf = t & 1;
    if (t + 1 < nk) load((t + 1) * SB_K);  // in flight while this tile is multiplied
#pragma unroll
    for (int k = 0; k < SB_K; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
      float a[8], bv[8];
      a[0] = a0.x, a[1] = a0.y, a[2] = a0.z, a[3] = a0.w, a[4] = a1.x, a[5] = a1.y, a[6] = a1.z, a[7] = a1.w;
      bv[0] = b0.x, bv[1] = b0.y, bv[2] = b0.z, bv[3] = b0.w, bv[4] = b1.x, bv[5] = b1.y, bv[6] = b1.z, bv[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
    }
    if (t + 1 < nk) store(buf ^ 1);  // the other buffer was last read before the previous barrier
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias != nullptr) v += ld_f32(bias + (bias_m ? gm : gn));
      st_f32(C + gm * ldc + gn, v);
      for (int q = 0; q < peers.n; ++q) st_f32(static_cast<T*>(peers.base[q]) + bz * sc + gm * ldc + gn, v);
    }
  }
}

template <typename T>
__global__ void fill_bias_kernel(T* __restrict__ C, const T* __restrict__ bias, long long M, long long N,
                                 long long ldc, long long sc, int bias_m, PeerOut peers) {
  const long long bz = blockIdx.y;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < M * N; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / N, c = i - r * N;
    const float v = bias != nullptr ? ld_f32(bias + (bias_m ? r : c)) : 0.0f;
    st_f32(C + bz * sc + r * ldc + c, v);
    for (int q = 0; q < peers.n; ++q) st_f32(static_cast<T*>(peers.base[q]) + bz * sc + r * ldc + c, v);
  }
}

// C[r, c] += bias[c]: blockIdx.x / threadIdx.x pick the column (the bias
// value stays in a register), blockIdx.y strides over rows; no index division.
template <typename T>
__global__ void add_bias_kernel(T* __restrict__ C, const T* __restrict__ bias, long long rows, long long cols) {
  const long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const float b = ld_f32(bias + c);
  for (long long r = blockIdx.y; r < rows; r += gridDim.y) {
    T* p = C + r * cols + c;
    st_f32(p, ld_f32(p) + b);
  }
}

template <typename T>
cudaError_t simt_t(const Gemm& g, cudaStream_t s) {
  dim3 grid(unsigned((g.N + SB_N - 1) / SB_N), unsigned((g.M + SB_M - 1) / SB_M), unsigned(g.batch));
  gemm_simt_kernel<T><<<grid, 256, 0, s>>>(reinterpret_cast<const T*>(g.A), reinterpret_cast<const T*>(g.B),
                                           reinterpret_cast<T*>(g.C), reinterpret_cast<const T*>(g.bias), int(g.M),
                                           int(g.N), int(g.K), g.lda, g.ldb, g.ldc, g.sa, g.sb, g.sc, g.b_kmajor,
                                           g.bias_m, g.peers);
  return cudaGetLastError();
}

template <typename T>
cudaError_t fill_t(const Gemm& g, cudaStream_t s) {
  long long blocks = (g.M * g.N + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  fill_bias_kernel<T><<<dim3(unsigned(blocks), unsigned(g.batch)), 256, 0, s>>>(
      reinterpret_cast<T*>(g.C), reinterpret_cast<const T*>(g.bias), g.M, g.N, g.ldc, g.sc, g.bias_m, g.peers);
  return cudaGetLastError();
}

template <typename T>
cudaError_t bias_t(void* C, const void* bias, int64_t rows, int64_t cols, cudaStream_t s) {
  const long long bx = (cols + 255) / 256;
  if (bx > 0x7fffffffLL) return cudaErrorInvalidValue;
  long long by = (8192 + bx - 1) / bx;  // about 8192 blocks in all
  if (by > rows) by = rows;
  if (by > 65535) by = 65535;
  if (by < 1) by = 1;
  add_bias_kernel<T><<<dim3(unsigned(bx), unsigned(by)), 256, 0, s>>>(reinterpret_cast<T*>(C),
                                                                      reinterpret_cast<const T*>(bias), rows, cols);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_simt(const Gemm& g, cudaStream_t s) {
  switch (g.dtype) {
    case CMPX_F16: return simt_t<__half>(g, s);
    case CMPX_BF16: return simt_t<__nv_bfloat16>(g, s);
    default: return simt_t<float>(g, s);
  }
}

cudaError_t launch_fill_bias(const Gemm& g, cudaStream_t s) {
  switch (g.dtype) {
    case CMPX_F16: return fill_t<__half>(g, s);
    case CMPX_BF16: return fill_t<__nv_bfloat16>(g, s);
    default: return fill_t<float>(g, s);
  }
}

cudaError_t launch_add_bias(int dtype, void* C, const void* bias, int64_t rows, int64_t cols, cudaStream_t s) {
  switch (dtype) {
    case CMPX_F16: return bias_t<__half>(C, bias, rows, cols, s);
    case CMPX_BF16: return bias_t<__nv_bfloat16>(C, bias, rows, cols, s);
    default: return bias_t<float>(C, bias, rows, cols, s);
  }
}

}  // namespace cmpx
