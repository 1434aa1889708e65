// ref_shim.cu -- extern "C" entry points over the reference's own launchers.
//
// TEST INFRASTRUCTURE ONLY.  Linked together with the reference's unmodified
// src/cuda/{fp16,fp32,bf16}_matmul.cu (compiled from /root/reference by
// oracle/Makefile into oracle/_ref/libref_matmul.so) so the GPU parity tests
// can run the reference kernel itself on the B200 as a second oracle.  The
// launcher prototypes are the reference's (src/main.cpp:12-19).
#include <cuda_runtime.h>

void launch_matmul_fp16(const void* input, const void* weight, void* output, int M, int N, int K);
void launch_matmul_fp32(const float* input, const float* weight, float* output, int M, int N, int K);
void launch_matmul_bf16(const void* input, const void* weight, void* output, int M, int N, int K);

// dtype: 0 = fp16, 1 = bf16, 2 = fp32.  Launches on the legacy default stream
// (as the reference does), waits for completion, returns the cudaError_t.
extern "C" __attribute__((visibility("default"))) int ref_matmul(int dtype, const void* A, const void* B, void* C,
                                                                  int M, int N, int K) {
  cudaGetLastError();
  if (dtype == 0) launch_matmul_fp16(A, B, C, M, N, K);
  else if (dtype == 1) launch_matmul_bf16(A, B, C, M, N, K);
  else launch_matmul_fp32(static_cast<const float*>(A), static_cast<const float*>(B), static_cast<float*>(C), M, N, K);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaGetLastError();
  return int(e);
}
