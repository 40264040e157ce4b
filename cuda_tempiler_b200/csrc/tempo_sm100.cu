// Host side of the sm_100a GEMM backend: TMA descriptor construction, the M-ladder
// dispatcher, the split-K cost model and the extern "C" entry points declared in
// include/tempo_sm100.h.  The dispatch contract mirrors the reference's shipped launch()
// (kernels/shipped/gemm_fp16/sm_70/launch.cuh:32-75, dispatch.inc:15-26): applicable()
// guards the layout, the ladder picks an instantiation, and cudaErrorInvalidConfiguration
// means "not covered, take your fallback".
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "tempo_sm100.h"
#include "launch.cuh"
#include "elementwise.cuh"
#include "collective.cuh"

namespace tempo_sm100 {
namespace {

struct LadderRow {
  int m_max;  // inclusive upper bound on M (0x7fffffff = everything else)
  int bn, swap, group_m;
  int cta_group;  // 1, or 2 for the 2-CTA 256 x BN prefill tiles (fp16)
};

#include "gemm_fp16/sm_100a/dispatch.inc"
#include "gemm_w8a16/sm_100a/dispatch.inc"

const LadderRow* ladder_row(int wkind, int M) {
  const LadderRow* rows = wkind == 0 ? kLadderFp16 : kLadderW8;
  const int n = wkind == 0 ? (int)(sizeof(kLadderFp16) / sizeof(LadderRow))
                           : (int)(sizeof(kLadderW8) / sizeof(LadderRow));
  for (int i = 0; i < n; ++i)
    if (M <= rows[i].m_max) return &rows[i];
  return nullptr;
}

// Cycle model of one launch, used to pick the k-split (mirrored by the shipped select.py):
//   SM side:  ceil(units / SMs) waves x (k-blocks per unit x per-k-block + split fix-up).
//             Per k-block = max(MMA, operand feed): one 128xBNx16 UMMA costs max(BN/2 tensor
//             cycles, (128+BN)*32 B / 128 B-per-cycle shared-memory reads); the feed is
//             (128+BN)*128 B per k-block at ~100 B/cycle/SM from L2.  The split fix-up writes
//             and re-reads a 128xBN fp32 slice (charged 3x for the counter/barrier).
//   HBM side: compulsory bytes (2MK + w_b NK + 2MN) at ~3400 B/cycle for the whole GPU.
//   launch:   the larger of the two.
// Cycle model of one launch (the busiest SM): waves of units, each k-block costing the larger
// of its UMMAs and its operand feed -- weight bytes stream from HBM at about 32 B/cycle per SM
// (measured TMA streaming rate), activation bytes from L2 at about 100 -- plus the k-split
// fixup: ~1500 cycles through distributed shared memory (splits <= kMaxClusterSplit), the
// fp32 partial round trip through global memory beyond; never below the HBM time.
double launch_cycles(int tiles, int num_kb, int sms, int bn, int swap, int wbytes, int s,
                     double hbm_bytes) {
  const long long units = (long long)tiles * s;
  const long long waves = (units + sms - 1) / sms;
  const double mma = 4.0 * std::max(bn / 2.0, (128.0 + bn) / 4.0);
  const double w_rows = swap ? 128.0 : bn, a_rows = swap ? bn : 128.0;
  const double feed = w_rows * 64.0 * wbytes / 32.0 + a_rows * 128.0 / 100.0;
  const double kb = (double)((num_kb + s - 1) / s);
  const double fixup = s == 1 ? 0.0
                     : s <= kMaxClusterSplit ? 1500.0
                                             : 3.0 * 128.0 * bn * 4.0 / 100.0 + 1500.0;
  const double sm_side = (double)waves * (kb * std::max(mma, feed) + fixup);
  return std::max(sm_side, hbm_bytes / 3400.0);
}

int choose_splits(int tiles, int num_kb, int sms, int bn, int swap, int wbytes, size_t ws_bytes,
                  double hbm_bytes) {
  if (sms <= 0) return 1;
  int best = 1;
  double best_c = launch_cycles(tiles, num_kb, sms, bn, swap, wbytes, 1, hbm_bytes);
  // the dispatcher keeps to cluster k-splits (the global-workspace path stays reachable as
  // an explicit hyperform)
  const int smax = std::min(kMaxClusterSplit, num_kb / 2);
  for (int s = 2; s <= smax; ++s) {
    if (ws_needed(tiles, s, bn) > ws_bytes) break;
    // a cluster k-split launch is one CTA per unit, not persistent: one wave only
    if (s <= kMaxClusterSplit && (long long)tiles * s > sms) continue;
    const double c = launch_cycles(tiles, num_kb, sms, bn, swap, wbytes, s, hbm_bytes);
    if (c < best_c * 0.97) {
      best = s;
      best_c = c;
    }
  }
  return best;
}

bool select_hyper(int wkind, int M, int N, int K, size_t ws_bytes, Hyper& h, int sms) {
  const LadderRow* r = ladder_row(wkind, M);
  if (!r) return false;
  h.bn = r->bn;
  h.swap = r->swap;
  h.group_m = r->group_m;
  h.max_ctas = 0;
  h.cta_group = (wkind == 0 && r->cta_group == 2 && !r->swap) ? 2 : 1;
  const int rows_p = h.swap ? N : M, rows_q = h.swap ? M : N;
  // a 128-wide 1-CTA row whose tiles overflow one wave takes the 256-wide tile (half the
  // activation re-reads, one wave) when that instantiation exists
  if (h.cta_group == 1 && !h.swap && h.bn == 128 && sms > 0 &&
      (long long)((rows_p + 127) / 128) * ((rows_q + 127) / 128) > sms &&
      find_inst(wkind, 256, 0) != nullptr)
    h.bn = 256;
  const int tiles = ((rows_p + 127) / 128) * ((rows_q + std::max(h.bn, 1) - 1) / std::max(h.bn, 1));
  const int num_kb = (K + 63) / 64;
  if (h.bn == 0) {  // streaming GEMV row of the ladder
    h.splits = 1;
    return M <= kGemvMaxM;
  }
  if (h.cta_group == 2) {  // pair tiles: width and split tail by the wave model
    h.bn = choose_pair_bn(M, N, K, sms, h.bn, ws_bytes);
    h.splits = 2;
    return h.bn != 0;
  }
  const double hbm = 2.0 * M * K + (wkind == 0 ? 2.0 : 1.0) * N * K + 2.0 * M * N;
  h.splits = choose_splits(tiles, num_kb, sms, h.bn, h.swap, wkind == 0 ? 2 : 1, ws_bytes, hbm);
  return find_inst(wkind, h.bn, h.swap) != nullptr;
}

// Workspace bytes a hyperform needs (0: none) and, in *zero_bytes, how many leading bytes of it
// are arrival counters that must be zero before a launch.
size_t hyper_ws(int M, int N, int K, const Hyper& h, int sms, size_t ws_cap, size_t* zero_bytes) {
  if (h.cta_group == 2) {
    const PairPlan pl = pair_plan(M, N, K, h.bn, sms, h.max_ctas, h.splits > 1, ws_cap);
    if (zero_bytes)
      *zero_bytes = pl.ws_bytes ? counters_used_bytes(2 * (pl.tiles - pl.sk_tile0)) : 0;
    return pl.ws_bytes;
  }
  const int rows_p = h.swap ? N : M, rows_q = h.swap ? M : N;
  const int bn = std::max(h.bn, 1);
  const int tiles = ((rows_p + 127) / 128) * ((rows_q + bn - 1) / bn);
  const size_t need = h.bn == 0 ? 0 : ws_needed(tiles, h.splits, h.bn);
  if (zero_bytes) *zero_bytes = need ? counters_used_bytes(tiles) : 0;
  return need;
}

cudaError_t run(const Problem& pr, const Hyper& h, cudaStream_t st) {
  if (h.bn == 0) return run_gemv(pr, st, h.group_m);
  if (h.cta_group == 2) return run_pair(pr, h, st);
  const InstEntry* e = find_inst(pr.wkind, h.bn, h.swap);
  if (!e) return cudaErrorInvalidConfiguration;
  return e->fn(pr, h, st);
}

int current_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return dev_info(dev).sms;
}

}  // namespace
}  // namespace tempo_sm100

using namespace tempo_sm100;

extern "C" {

int tempo_sm100_gemm_fp16_applicable(const void* A, const void* B, const void* C, int M, int N,
                                     int K, int lda, int ldb, int ldc) {
  return fp16_applicable(A, B, C, M, N, K, lda, ldb, ldc) ? 1 : 0;
}

int tempo_sm100_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                          int ldb, int ldc, void* ws, size_t ws_bytes, void* stream) {
  if (!fp16_applicable(A, B, C, M, N, K, lda, ldb, ldc)) return cudaErrorInvalidConfiguration;
  if (ws && !aligned16(ws)) return cudaErrorInvalidValue;  // counters, fp32 partials
  Hyper h{};
  if (!select_hyper(0, M, N, K, ws ? ws_bytes : 0, h, current_sms()))
    return cudaErrorInvalidConfiguration;
  Problem pr{0, A, B, nullptr, nullptr, C, M, N, K, lda, ldb, ldc, 0, ws, ws_bytes};
  return run(pr, h, static_cast<cudaStream_t>(stream));
}

int tempo_sm100_gemm_w8a16_applicable(const void* A, const void* W, const void* scale,
                                      const void* zero, const void* C, int M, int N, int K,
                                      int lda, int ldw, int ldc, int quant_kind, int group_size) {
  return w8_applicable(A, W, scale, zero, C, M, N, K, lda, ldw, ldc, quant_kind, group_size) ? 1
                                                                                              : 0;
}

int tempo_sm100_gemm_w8a16(const void* A, const void* W, const void* scale, const void* zero,
                           void* C, int M, int N, int K, int lda, int ldw, int ldc, int quant_kind,
                           int group_size, void* ws, size_t ws_bytes, void* stream) {
  if (!w8_applicable(A, W, scale, zero, C, M, N, K, lda, ldw, ldc, quant_kind, group_size))
    return cudaErrorInvalidConfiguration;
  // the expanded weights are written with 16-byte stores from the start of ws
  if (ws && !aligned16(ws)) return cudaErrorInvalidValue;
  const int sms = current_sms();
  if (M >= kExpandMinM && ws) {
    // expanded weights at the front of the workspace, the fp16 launch's workspace behind them
    const size_t wexp = expand_ws_bytes(N, K);
    Hyper hf{};
    if (ws_bytes >= wexp && select_hyper(0, M, N, K, ws_bytes - wexp, hf, sms)) {
      cudaStream_t st = static_cast<cudaStream_t>(stream);
      Problem pw{quant_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, wexp};
      __half* wf = static_cast<__half*>(ws);
      cudaError_t e = launch_expand(pw, wf, st);
      if (e != cudaSuccess) return e;
      Problem pr{0, A, wf, nullptr, nullptr, C, M, N, K, lda, K, ldc, 0,
                 static_cast<char*>(ws) + wexp, ws_bytes - wexp};
      return run(pr, hf, st);
    }
  }
  Hyper h{};
  if (!select_hyper(quant_kind, M, N, K, ws ? ws_bytes : 0, h, current_sms()))
    return cudaErrorInvalidConfiguration;
  Problem pr{quant_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  return run(pr, h, static_cast<cudaStream_t>(stream));
}

size_t tempo_sm100_workspace_bytes(int M, int N, int K, int weight_kind) {
  Hyper h{};
  const int sms = current_sms();
  if (weight_kind != 0 && M >= kExpandMinM && (K % 16) == 0) {  // expanded weights + fp16 launch
    if (!select_hyper(0, M, N, K, (size_t)1 << 40, h, sms)) return 0;
    return expand_ws_bytes(N, K) + hyper_ws(M, N, K, h, sms, (size_t)1 << 40, nullptr);
  }
  if (!select_hyper(weight_kind, M, N, K, (size_t)1 << 40, h, sms)) return 0;
  return hyper_ws(M, N, K, h, sms, (size_t)1 << 40, nullptr);
}

int tempo_sm100_gemm_hyperform(int weight_kind, const void* A, const void* W, const void* scale,
                               const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                               int ldc, int group_size, int bn, int swap, int splits, int group_m,
                               int max_ctas, void* ws, size_t ws_bytes, void* stream) {
  if (weight_kind == 0) {
    if (!fp16_applicable(A, W, C, M, N, K, lda, ldw, ldc)) return cudaErrorInvalidConfiguration;
  } else if (!w8_applicable(A, W, scale, zero, C, M, N, K, lda, ldw, ldc, weight_kind,
                            group_size)) {
    return cudaErrorInvalidConfiguration;
  }
  if (swap < 0 || swap > 2) return cudaErrorInvalidConfiguration;
  Hyper h{bn, swap, splits < 1 ? 1 : splits, group_m < 1 ? 1 : group_m, max_ctas};
  Problem pr{weight_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  return run(pr, h, static_cast<cudaStream_t>(stream));
}

int tempo_sm100_gemm_hyperform_cg(int weight_kind, const void* A, const void* W, const void* scale,
                                  const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                                  int ldc, int group_size, int bn, int swap, int splits,
                                  int group_m, int max_ctas, int cta_group, void* ws,
                                  size_t ws_bytes, void* stream) {
  if (cta_group != 2)
    return tempo_sm100_gemm_hyperform(weight_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc,
                                      group_size, bn, swap, splits, group_m, max_ctas, ws, ws_bytes,
                                      stream);
  if (weight_kind != 0 || swap) return cudaErrorInvalidConfiguration;
  if (!fp16_applicable(A, W, C, M, N, K, lda, ldw, ldc)) return cudaErrorInvalidConfiguration;
  Hyper h{bn, 0, splits > 1 ? 2 : 1, group_m < 1 ? 1 : group_m, max_ctas};
  h.cta_group = 2;
  Problem pr{0, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  return run(pr, h, static_cast<cudaStream_t>(stream));
}

int tempo_sm100_pair_resources(int bn, int* out6) { return pair_resources(bn, out6); }

int tempo_sm100_select(int weight_kind, int M, int N, int K, size_t ws_bytes, int* out5) {
  Hyper h{};
  const int sms = current_sms();
  if (weight_kind != 0 && M >= kExpandMinM && ws_bytes >= expand_ws_bytes(N, K) &&
      select_hyper(0, M, N, K, ws_bytes - expand_ws_bytes(N, K), h, sms)) {
    weight_kind = 0;  // expanded weights: the fp16 launch's configuration
  } else if (!select_hyper(weight_kind, M, N, K, ws_bytes, h, sms)) {
    return cudaErrorInvalidConfiguration;
  }
  const InstEntry* e = find_inst(weight_kind, h.bn, h.swap);
  if (out5) {
    out5[0] = h.bn;
    out5[1] = h.swap;
    out5[2] = h.splits;
    out5[3] = h.group_m;
    out5[4] = e ? e->stages : 0;
  }
  return 0;
}

int tempo_sm100_hyperform_resources(int weight_kind, int bn, int swap, int* out6) {
  const InstEntry* e = find_inst(weight_kind, bn, swap);
  if (!e) return cudaErrorInvalidConfiguration;
  cudaFuncAttributes fa{};
  cudaError_t err = cudaFuncGetAttributes(&fa, e->kern);
  if (out6) {
    out6[0] = e->threads;
    out6[1] = e->smem;
    out6[2] = e->stages;
    out6[3] = e->tmem_cols;
    out6[4] = err == cudaSuccess ? fa.numRegs : -1;
    out6[5] = err == cudaSuccess ? (int)fa.localSizeBytes : -1;
  }
  return err;
}

int tempo_sm100_naive_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K,
                                int lda, int ldb, int ldc, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !C) return cudaErrorInvalidValue;
  return launch_naive_fp16(static_cast<const __half*>(A), static_cast<const __half*>(B),
                           static_cast<__half*>(C), M, N, K, lda, ldb, ldc,
                           static_cast<cudaStream_t>(stream));
}

int tempo_sm100_naive_gemm_w8a16(const void* A, const void* W, const void* scale,
                                 const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                                 int ldc, int quant_kind, int group_size, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !W || !C || !scale) return cudaErrorInvalidValue;
  if (quant_kind == TEMPO_W8_UINT8_GROUP && (!zero || group_size <= 0 || K % group_size))
    return cudaErrorInvalidValue;
  if (quant_kind != TEMPO_W8_INT8_PER_CHANNEL && quant_kind != TEMPO_W8_UINT8_GROUP)
    return cudaErrorInvalidValue;
  return launch_naive_w8a16(static_cast<const __half*>(A), static_cast<const uint8_t*>(W),
                            static_cast<const __half*>(scale), static_cast<const uint8_t*>(zero),
                            static_cast<__half*>(C), M, N, K, lda, ldw, ldc, quant_kind,
                            group_size, static_cast<cudaStream_t>(stream));
}

int tempo_sm100_silu_mul(const void* gu, void* out, int M, int I, int ld_gu, int ld_out,
                         int block, void* stream) {
  if (M <= 0 || I <= 0 || (I % 8) || (ld_gu % 8) || (ld_out % 8) || ld_gu < 2 * I || ld_out < I)
    return cudaErrorInvalidValue;
  if (block < 0 || (block && ((block % 8) || (I % block)))) return cudaErrorInvalidValue;
  if (!aligned16(gu) || !aligned16(out)) return cudaErrorInvalidValue;
  return launch_silu_mul(static_cast<const __half*>(gu), static_cast<__half*>(out), M, I, ld_gu,
                         ld_out, block, static_cast<cudaStream_t>(stream));
}

int tempo_sm100_gemm_fp16_swiglu(const void* A, const void* W, void* C, int M, int N, int K,
                                 int lda, int ldw, int ldc, void* stream) {
  if (M <= kSwigluMinM || N % 128 || !fp16_applicable(A, W, C, M, N / 2, K, lda, ldw, ldc))
    return cudaErrorInvalidConfiguration;
  if (ldw < K || (ldw % 8)) return cudaErrorInvalidConfiguration;
  Problem pr{0, A, W, nullptr, nullptr, C, M, N, K, lda, ldw, ldc, 0, nullptr, 0};
  return run_pair_swiglu(pr, current_sms(), static_cast<cudaStream_t>(stream));
}

int tempo_sm100_gemm_w8a16_swiglu(const void* A, const void* W, const void* scale,
                                  const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                                  int ldc, int quant_kind, int group_size, void* ws,
                                  size_t ws_bytes, void* stream) {
  if (M < kExpandMinM || N % 128 || !ws || ws_bytes < expand_ws_bytes(N, K))
    return cudaErrorInvalidConfiguration;
  if (!aligned16(ws)) return cudaErrorInvalidValue;
  if (!w8_applicable(A, W, scale, zero, C, M, N, K, lda, ldw, N, quant_kind, group_size) ||
      ldc < N / 2 || (ldc % 8))
    return cudaErrorInvalidConfiguration;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Problem pw{quant_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  __half* wf = static_cast<__half*>(ws);
  cudaError_t e = launch_expand(pw, wf, st);
  if (e != cudaSuccess) return e;
  Problem pr{0, A, wf, nullptr, nullptr, C, M, N, K, lda, K, ldc, 0, nullptr, 0};
  return run_pair_swiglu(pr, current_sms(), st);
}

int tempo_sm100_ipc_alloc(size_t bytes, void** out_ptr) {
  if (!out_ptr || bytes == 0) return cudaErrorInvalidValue;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return e;
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return e;
  }
  *out_ptr = p;
  return cudaSuccess;
}

int tempo_sm100_ipc_free(void* ptr) { return cudaFree(ptr); }

int tempo_sm100_ipc_handle(const void* dptr, void* out_handle) {
  if (!dptr || !out_handle) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dptr));
  if (e == cudaSuccess) std::memcpy(out_handle, &h, sizeof(h));
  return e;
}

int tempo_sm100_ipc_open(const void* handle, void** out_ptr) {
  if (!handle || !out_ptr) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

int tempo_sm100_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr); }

int tempo_sm100_allreduce_oneshot_timed(const void* src, void* dst, long long n, long long cap,
                                        void* const* recv, void* const* flags, int tp, int rank,
                                        unsigned epoch, int ctas, unsigned long long wait_ns,
                                        void* stream) {
  if (!src || !dst || !recv || !flags || tp < 1 || tp > kArMaxTp || rank < 0 || rank >= tp)
    return cudaErrorInvalidValue;
  if (n <= 0 || (n % 8) || n > cap || (cap % 8) || ctas < 1 || ctas > kArMaxCtas || epoch == 0)
    return cudaErrorInvalidValue;
  if (wait_ns == 0 || wait_ns > kWaitLimitNs) return cudaErrorInvalidValue;
  if (!aligned16(src) || !aligned16(dst)) return cudaErrorInvalidValue;
  PeerSet ps{};
  for (int p = 0; p < tp; ++p) {
    if (!recv[p] || !flags[p] || !aligned16(recv[p])) return cudaErrorInvalidValue;
    ps.recv[p] = static_cast<__half*>(recv[p]);
    ps.flags[p] = static_cast<uint32_t*>(flags[p]);
  }
  return launch_ex(k_allreduce_oneshot, dim3(ctas), dim3(256), 0,
                   static_cast<cudaStream_t>(stream), 1, static_cast<const __half*>(src),
                   static_cast<__half*>(dst), n, cap, ps, tp, rank, (uint32_t)epoch, wait_ns);
}

int tempo_sm100_allreduce_oneshot(const void* src, void* dst, long long n, long long cap,
                                  void* const* recv, void* const* flags, int tp, int rank,
                                  unsigned epoch, int ctas, void* stream) {
  return tempo_sm100_allreduce_oneshot_timed(src, dst, n, cap, recv, flags, tp, rank, epoch, ctas,
                                             kWaitLimitNs, stream);
}

int tempo_sm100_device_status(int* out4, int reset) {
  int h[4] = {0, 0, 0, 0};
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(h, g_status, sizeof(h));
  if (e != cudaSuccess) return e;
  if (out4) std::memcpy(out4, h, sizeof(h));
  if (reset) {
    const int z[4] = {0, 0, 0, 0};
    e = cudaMemcpyToSymbol(g_status, z, sizeof(z));
  }
  return e;
}

const char* tempo_sm100_version(void) { return "tempo-sm100 0.1 (sm_100a, tcgen05/TMA)"; }

}  // extern "C"

// ==========================================================================================
// Allocation-free entry point: the fp16 GEMM with its split-K scratch in a static device array.
//
// Some callers cannot allocate device memory for us: serving frameworks that reserve almost all
// of HBM up front for their own caching allocator (a foreign cudaMalloc then fails or
// fragments their pool), latency-critical paths where cudaMalloc/cudaFree would implicitly
// synchronise the device, and thin FFI callers that have no device allocator to hand us a
// workspace.  For them the split-K partials and tile counters live in the fixed array below.
// It is part of the module image, so every GPU that loads this library holds
// TEMPO_SM100_NOALLOC_SCRATCH_BYTES of it until the process exits.
// ==========================================================================================
static __device__ __align__(256) unsigned char tempo_noalloc_scratch[TEMPO_SM100_NOALLOC_SCRATCH_BYTES];

namespace {
std::once_flag g_noalloc_once[tempo_sm100::kMaxDevices];
cudaError_t g_noalloc_err[tempo_sm100::kMaxDevices];
void* g_noalloc_ptr[tempo_sm100::kMaxDevices];
}  // namespace

extern "C" int tempo_sm100_gemm_fp16_noalloc(const void* A, const void* B, void* C, int M, int N,
                                             int K, int lda, int ldb, int ldc, void* stream) {
  using namespace tempo_sm100;
  if (!fp16_applicable(A, B, C, M, N, K, lda, ldb, ldc)) return cudaErrorInvalidConfiguration;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  // First call on a device (that device current): resolve the device address of the array.
  // In host code `tempo_noalloc_scratch` is only a host-side stand-in, never a device pointer.
  std::call_once(g_noalloc_once[dev], [dev] {
    void* p = nullptr;
    g_noalloc_err[dev] = cudaGetSymbolAddress(&p, tempo_noalloc_scratch);
    g_noalloc_ptr[dev] = g_noalloc_err[dev] == cudaSuccess ? p : nullptr;
  });
  if (g_noalloc_err[dev] != cudaSuccess) return g_noalloc_err[dev];
  void* scratch = g_noalloc_ptr[dev];

  // Same choice as tempo_sm100_gemm_fp16 given a workspace of tempo_sm100_workspace_bytes.
  Hyper h{};
  const int sms = current_sms();
  if (!select_hyper(0, M, N, K, (size_t)1 << 40, h, sms)) return cudaErrorInvalidConfiguration;
  size_t zero_bytes = 0;
  const size_t need = hyper_ws(M, N, K, h, sms, (size_t)1 << 40, &zero_bytes);
  if (need > (size_t)TEMPO_SM100_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (need > 0) {
    // The counters must start at zero; the array keeps whatever the previous call left.
    e = cudaMemsetAsync(scratch, 0, zero_bytes, st);
    if (e != cudaSuccess) return e;
  }
  Problem pr{0, A, B, nullptr, nullptr, C, M, N, K, lda, ldb, ldc, 0, scratch,
             (size_t)TEMPO_SM100_NOALLOC_SCRATCH_BYTES};
  return run(pr, h, st);
}
