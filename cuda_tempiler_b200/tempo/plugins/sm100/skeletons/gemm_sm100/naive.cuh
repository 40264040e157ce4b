// The naive INPUT bar: one thread per output element, fp32 accumulation, 16x16 CTAs.  This is
// the operation of the reference's declared input kernel (kernels/naive/gemm_fp16.cu:60-76,
// C[m][n] = sum_k A[m][k] * B[n][k]) and its W8A16 analogue (no naive W8A16 input exists in
// the reference; this one dequantises each weight in fp32 on the fly).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tempo_sm100 {

__global__ void k_naive_fp16(const __half* __restrict__ A, const __half* __restrict__ B,
                             __half* __restrict__ C, int M, int N, int K, long long lda,
                             long long ldb, long long ldc) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y * blockDim.y + threadIdx.y;
  if (m >= M || n >= N) return;
  const __half* a = A + (long long)m * lda;
  const __half* b = B + (long long)n * ldb;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) acc += __half2float(a[k]) * __half2float(b[k]);
  C[(long long)m * ldc + n] = __float2half_rn(acc);
}

__global__ void k_naive_w8a16(const __half* __restrict__ A, const uint8_t* __restrict__ W,
                              const __half* __restrict__ scale, const uint8_t* __restrict__ zero,
                              __half* __restrict__ C, int M, int N, int K, long long lda,
                              long long ldw, long long ldc, int kind, int group) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y * blockDim.y + threadIdx.y;
  if (m >= M || n >= N) return;
  const __half* a = A + (long long)m * lda;
  const uint8_t* w = W + (long long)n * ldw;
  float acc = 0.f;
  if (kind == 1) {
    for (int k = 0; k < K; ++k) acc += __half2float(a[k]) * (float)(int8_t)w[k];
    acc *= __half2float(scale[n]);
  } else {
    for (int k = 0; k < K; ++k) {
      const int g = k / group;  // scale and zero are [K/group][N]
      const float s = __half2float(scale[(long long)g * N + n]);
      const float z = (float)zero[(long long)g * N + n];
      acc += __half2float(a[k]) * (((float)w[k] - z) * s);
    }
  }
  C[(long long)m * ldc + n] = __float2half_rn(acc);
}

inline cudaError_t launch_naive_fp16(const __half* A, const __half* B, __half* C, int M, int N,
                                     int K, long long lda, long long ldb, long long ldc,
                                     cudaStream_t st) {
  const dim3 blk(16, 16), grid((N + 15) / 16, (M + 15) / 16);
  k_naive_fp16<<<grid, blk, 0, st>>>(A, B, C, M, N, K, lda, ldb, ldc);
  return cudaGetLastError();
}

inline cudaError_t launch_naive_w8a16(const __half* A, const uint8_t* W, const __half* scale,
                                      const uint8_t* zero, __half* C, int M, int N, int K,
                                      long long lda, long long ldw, long long ldc, int kind,
                                      int group, cudaStream_t st) {
  const dim3 blk(16, 16), grid((N + 15) / 16, (M + 15) / 16);
  k_naive_w8a16<<<grid, blk, 0, st>>>(A, W, scale, zero, C, M, N, K, lda, ldw, ldc, kind, group);
  return cudaGetLastError();
}

}  // namespace tempo_sm100
