// Elementwise kernels the tensor-parallel MLP needs between its two GEMMs.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tempo_sm100 {

// out[m][i] = silu(gate) * up for one gate_up GEMM output row m.  block 0: the row holds the
// gate half [0, I) and the up half [I, 2I); block b > 0: gate and up alternate in blocks of b
// columns (gate i at (i / b) 2b + i % b, its up b columns later).  8 halves per thread with
// 16-byte loads and stores (I and b multiples of 8).
__global__ void k_silu_mul(const __half* __restrict__ gu, __half* __restrict__ out, int M, int I,
                           long long ld_gu, long long ld_out, int block) {
  const long long vec = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = I / 8;
  if (vec >= (long long)M * per_row) return;
  const int m = (int)(vec / per_row);
  const int i = (int)(vec % per_row) * 8;
  const int gi = block ? (i / block) * 2 * block + i % block : i;
  const int ui = gi + (block ? block : I);
  const uint4 g = *reinterpret_cast<const uint4*>(gu + m * ld_gu + gi);
  const uint4 u = *reinterpret_cast<const uint4*>(gu + m * ld_gu + ui);
  const __half2* gh = reinterpret_cast<const __half2*>(&g);
  const __half2* uh = reinterpret_cast<const __half2*>(&u);
  uint4 o;
  __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 x = __half22float2(gh[j]);
    const float2 y = __half22float2(uh[j]);
    oh[j] = __floats2half2_rn(x.x / (1.f + expf(-x.x)) * y.x, x.y / (1.f + expf(-x.y)) * y.y);
  }
  *reinterpret_cast<uint4*>(out + m * ld_out + i) = o;
}

inline cudaError_t launch_silu_mul(const __half* gu, __half* out, int M, int I, long long ld_gu,
                                   long long ld_out, int block, cudaStream_t st) {
  const long long n = (long long)M * (I / 8);
  const int threads = 256;
  k_silu_mul<<<(unsigned)((n + threads - 1) / threads), threads, 0, st>>>(gu, out, M, I, ld_gu,
                                                                        ld_out, block);
  return cudaGetLastError();
}

}  // namespace tempo_sm100
