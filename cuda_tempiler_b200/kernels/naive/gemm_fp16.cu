// Naive INPUT kernel for the fp16 GEMM: the declared operation the tempolator recognises.
//
// TEMPO-OP: gemm
// dtype: a=fp16 b=fp16 c=fp16 acc=fp32
// layout: a=k b=k c=n
// shape: M=* N=* K=*
// tol_rel_l2: 3e-3
// entry: naive_gemm_fp16
// signature: (const __half* A, const __half* B, __half* C, int M, int N, int K)
// TEMPO-OP-END
//
// C[m][n] = sum_k A[m][k] * B[n][k]; one thread per output cell, fp32 accumulation.
#include <cuda_fp16.h>

__global__ void naive_gemm_fp16(const __half* A, const __half* B, __half* C, int M, int N, int K) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y * blockDim.y + threadIdx.y;
  if (m >= M || n >= N) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k)
    acc += __half2float(A[(long long)m * K + k]) * __half2float(B[(long long)n * K + k]);
  C[(long long)m * N + n] = __float2half_rn(acc);
}
