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

constexpr int SB_M = 64, SB_N = 64, SB_K = 16;

// 256 threads, each computes a 4x4 block of a 64x64 tile.  blockIdx.z = batch.
template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                        T* __restrict__ C, const T* __restrict__ bias, int M, int N,
                                                        int K, long long lda, long long ldb, long long ldc,
                                                        long long sa, long long sb, long long sc, int b_kmajor,
                                                        int bias_m, PeerOut peers) {
  __shared__ float As[SB_K][SB_M + 4];
  __shared__ float Bs[SB_K][SB_N + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * SB_M, n0 = blockIdx.x * SB_N;
  const long long bz = blockIdx.z;
  A += bz * sa;
  B += bz * sb;
  C += bz * sc;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += SB_K) {
    for (int i = tid; i < SB_M * SB_K; i += 256) {
      const int r = i / SB_K, k = i % SB_K;
      const int gm = m0 + r, gk = k0 + k;
      As[k][r] = (gm < M && gk < K) ? ld_f32(A + gm * lda + gk) : 0.0f;
    }
    for (int i = tid; i < SB_N * SB_K; i += 256) {
      int c, k;
      if (b_kmajor) {
        c = i / SB_K;
        k = i % SB_K;
      } else {
        k = i / SB_N;
        c = i % SB_N;
      }
      const int gn = n0 + c, gk = k0 + k;
      float v = 0.0f;
      if (gn < N && gk < K) v = b_kmajor ? ld_f32(B + gn * ldb + gk) : ld_f32(B + gk * ldb + gn);
      Bs[k][c] = v;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < SB_K; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
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
