// Frozen by the tempolator ship stage for gemm_w8a16 / sm_100a.  Do not edit: re-ship.
// The POD ABI of the shipped gemm_w8a16 kernels for sm_100a: C = A * W^T with 8-bit weights,
// fp16 activations and output, fp32 accumulation.  Same names and error contract as the
// gemm_fp16 POD (the reference's kernels/shipped/gemm_fp16/sm_70/launch.cuh:20-75 shape); the
// reference ships no W8A16 kernel (its sm70 skeleton tempo/plugins/sm70/skeletons/gemm_w8a16
// is unshipped), so the weight fields follow its GPTQ reconstruction formula
// (bench/gemm_baseline.py:214-231):
//
//   scale_kind TEMPO_W8_INT8_PER_CHANNEL  W int8 [N][K], scale fp16 [N]:        w = q * s[n]
//   scale_kind TEMPO_W8_UINT8_GROUP       W uint8 [N][K], scale fp16 [K/group][N],
//                                         zero uint8 [K/group][N]:  w = (q - z[g][n]) * s[g][n]
//
// The group-wise scale and zero arrays are GPTQ's own orientation (its scales array and the
// byte view of its qzeros, used as they are).  From M = 1024 on, given a workspace of at least
// N * K * 2 bytes, the weights are first expanded to fp16 in the workspace and the fp16 2-CTA
// tiles run on the copy (plan() reports expand = 1 and the bytes it wants).
#pragma once
#ifndef TEMPO_GEN_GEMM_W8A16_API
#define TEMPO_GEN_GEMM_W8A16_API

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#ifndef TEMPO_W8_INT8_PER_CHANNEL
#define TEMPO_W8_INT8_PER_CHANNEL 1
#define TEMPO_W8_UINT8_GROUP 2
#endif

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

struct W8A16Params {
  const __half* A;       // [M][K] fp16, row stride lda elements (multiple of 8)
  const uint8_t* W;      // [N][K] int8 or uint8, row stride ldw bytes (multiple of 16)
  const __half* scale;   // [N] or [K/group][N]
  const uint8_t* zero;   // [K/group][N] (group-wise only; NULL per-channel)
  __half* C;             // [M][N] fp16, row stride ldc elements (multiple of 8)
  int M, N, K;
  int lda, ldw, ldc;
  int scale_kind;        // TEMPO_W8_INT8_PER_CHANNEL or TEMPO_W8_UINT8_GROUP
  int group;             // group-wise: a multiple of 64 dividing K (ignored per-channel)
  void* ws = nullptr;    // workspace (16-byte aligned) or NULL
  size_t ws_bytes = 0;
};

inline bool shape_ok(const W8A16Params& p) {
  if (p.scale_kind != TEMPO_W8_INT8_PER_CHANNEL && p.scale_kind != TEMPO_W8_UINT8_GROUP)
    return false;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return false;
  if ((p.K % 16) || (p.N % 8)) return false;
  if (p.lda < p.K || p.ldw < p.K || p.ldc < p.N) return false;
  if ((p.lda % 8) || (p.ldw % 16) || (p.ldc % 8)) return false;
  if (p.scale_kind == TEMPO_W8_UINT8_GROUP &&
      (p.group <= 0 || (p.group % 64) || (p.K % p.group) || (p.N % 16)))
    return false;  // scale / zero rows are fetched by TMA: 16-byte row strides
  return true;
}

inline bool applicable(const W8A16Params& p) {
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!p.A || !p.W || !p.C || !p.scale) return false;
  if (!a16(p.A) || !a16(p.W) || !a16(p.C)) return false;
  if (p.scale_kind == TEMPO_W8_UINT8_GROUP && (!p.zero || !a16(p.scale) || !a16(p.zero)))
    return false;
  return shape_ok(p);
}

cudaError_t launch(const W8A16Params& p, cudaStream_t s);
cudaError_t plan(const W8A16Params& p, Choice* out);

}  // namespace gen
}  // namespace tempo

#endif  // TEMPO_GEN_GEMM_W8A16_API
