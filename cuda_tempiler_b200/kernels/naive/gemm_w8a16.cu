// Naive INPUT kernel for the W8A16 GEMM (no counterpart in the reference, whose W8A16
// skeleton was never shipped): uint8 weights with a group-wise fp16 scale and uint8 zero-point
// along K, W[n][k] = (q[n][k] - z[k/G][n]) * s[k/G][n] (the GPTQ reconstruction), fp16
// activations, fp32 accumulation.
//
// TEMPO-OP: gemm
// dtype: a=fp16 b=uint8 c=fp16 acc=fp32
// layout: a=k b=k c=n
// shape: M=* N=* K=*
// scale: group:128
// tol_rel_l2: 3e-3
// entry: naive_gemm_w8a16
// signature: (const __half* A, const unsigned char* W, const __half* S, const unsigned char* Z, __half* C, int M, int N, int K, int G)
// TEMPO-OP-END
#include <cuda_fp16.h>

__global__ void naive_gemm_w8a16(const __half* A, const unsigned char* W, const __half* S,
                                 const unsigned char* Z, __half* C, int M, int N, int K, int G) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y * blockDim.y + threadIdx.y;
  if (m >= M || n >= N) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) {
    const int g = k / G;
    const float w = ((float)W[(long long)n * K + k] - (float)Z[(long long)g * N + n]) *
                    __half2float(S[(long long)g * N + n]);
    acc += __half2float(A[(long long)m * K + k]) * w;
  }
  C[(long long)m * N + n] = __float2half_rn(acc);
}
