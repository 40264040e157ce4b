// Frozen by the tempolator ship stage for gemm_fp16 / sm_100a.  Do not edit: re-ship.
// The POD ABI of the shipped gemm_fp16 kernels for sm_100a -- the whole interface a host tree
// needs: plain pointers and ints, no framework types.  It replaces the reference's shipped
// kernels/shipped/gemm_fp16/sm_70/launch.cuh:20-75 (struct tempo::gen::GemmParams,
// applicable(), launch() defined in launch.cu whose body is dispatch.inc) with the same names
// and the same error contract:
//
//   cudaSuccess                      launched on the stream
//   cudaErrorInvalidConfiguration    not covered: take your own path (F.linear / cuBLAS)
//   anything else                    a real CUDA error
//
// Differences, both forced by the hardware path: a caller-owned split-K workspace (ws,
// ws_bytes; zero-filled once before first use, left zeroed by every launch; NULL is legal and
// means no split through global memory), and plan(), which reports the configuration launch()
// would run, and the workspace it wants, without launching anything.
#pragma once
#ifndef TEMPO_GEN_GEMM_FP16_API
#define TEMPO_GEN_GEMM_FP16_API

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace tempo {
namespace gen {

#ifndef TEMPO_GEN_CHOICE
#define TEMPO_GEN_CHOICE
// What a dispatch picks for one problem (filled by plan()).
struct Choice {
  int bn = 0;         // tile width (0: the streaming decode GEMV)
  int swap = 0;       // 0 plain tiles; 1 swap-AB (weights as the 128-row operand); 2 swap-AB
                      // with 8-bit weights dequantised in shared memory
  int splits = 1;     // k-split (2 on a 2-CTA row: a split tail is allowed)
  int group_m = 0;    // raster group (a GEMV's variant)
  int cta_group = 1;  // 2: 256 x bn tiles on 2-CTA clusters
  int expand = 0;     // W8A16: weights expanded to fp16 in ws first, then the fp16 tiles
  int stages = 0;     // pipeline depth of a 1-CTA tile instantiation (0 otherwise)
  size_t ws_bytes = 0;    // workspace this choice uses (0: none)
  size_t zero_bytes = 0;  // leading bytes of it that must be zero before the launch
};
#endif

// C[M][N] = A[M][K] * B[N][K]^T, fp16 in and out, fp32 accumulation.
struct GemmParams {
  const __half* A;  // [M][K], K contiguous, row stride lda elements
  const __half* B;  // [N][K], K contiguous, row stride ldb elements
  __half* C;        // [M][N], row stride ldc elements
  int M, N, K;
  int lda, ldb, ldc;        // in elements; multiples of 8 (16-byte TMA row strides)
  void* ws = nullptr;       // split-K workspace (16-byte aligned) or NULL
  size_t ws_bytes = 0;
};

// Shape and stride rules without the pointers (what plan() needs).
inline bool shape_ok(const GemmParams& p) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return false;
  if ((p.K % 8) || (p.N % 8)) return false;
  if (p.lda < p.K || p.ldb < p.K || p.ldc < p.N) return false;
  return !((p.lda % 8) || (p.ldb % 8) || (p.ldc % 8));
}

// false: not covered -- the caller takes its own path (the reference's applicable()).
inline bool applicable(const GemmParams& p) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!p.A || !p.B || !p.C || !a16(p.A) || !a16(p.B) || !a16(p.C)) return false;
  return shape_ok(p);
}

// Launch on `s`.  Defined in launch.cu, whose dispatch body is the generated dispatch.inc.
cudaError_t launch(const GemmParams& p, cudaStream_t s);

// The configuration launch(p, ...) would run given p.ws_bytes of workspace (p's pointers are
// not read); cudaErrorInvalidConfiguration when the problem is not covered.
cudaError_t plan(const GemmParams& p, Choice* out);

}  // namespace gen
}  // namespace tempo

#endif  // TEMPO_GEN_GEMM_FP16_API
