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
// The shipped artifacts, one translation unit: each op's launch.cu brings its POD ABI
// (launch.cuh), the frozen device code (kernel.cuh) and host layer -- both include-guarded, so
// the second op reuses the first's -- and tempo::gen::launch / plan around its generated
// dispatch.inc.  Every GEMM entry point below goes through tempo::gen.
#include "gemm_fp16/sm_100a/launch.cu"
#include "gemm_w8a16/sm_100a/launch.cu"
#include "elementwise.cuh"
#include "collective.cuh"

namespace tempo_sm100 {
namespace {

constexpr size_t kPlanAnyWorkspace = (size_t)1 << 40;

tempo::gen::GemmParams fp16_params(const void* A, const void* B, void* C, int M, int N, int K,
                                   int lda, int ldb, int ldc, void* ws, size_t ws_bytes) {
  tempo::gen::GemmParams p{static_cast<const __half*>(A), static_cast<const __half*>(B),
                           static_cast<__half*>(C), M, N, K, lda, ldb, ldc};
  p.ws = ws;
  p.ws_bytes = ws_bytes;
  return p;
}

tempo::gen::W8A16Params w8_params(const void* A, const void* W, const void* scale,
                                  const void* zero, void* C, int M, int N, int K, int lda,
                                  int ldw, int ldc, int kind, int group, void* ws,
                                  size_t ws_bytes) {
  tempo::gen::W8A16Params p{static_cast<const __half*>(A), static_cast<const uint8_t*>(W),
                            static_cast<const __half*>(scale), static_cast<const uint8_t*>(zero),
                            static_cast<__half*>(C), M, N, K, lda, ldw, ldc, kind, group};
  p.ws = ws;
  p.ws_bytes = ws_bytes;
  return p;
}

}  // namespace
}  // namespace tempo_sm100

using namespace tempo_sm100;

extern "C" {

int tempo_sm100_gemm_fp16_applicable(const void* A, const void* B, const void* C, int M, int N,
                                     int K, int lda, int ldb, int ldc) {
  return tempo::gen::applicable(fp16_params(A, B, const_cast<void*>(C), M, N, K, lda, ldb, ldc,
                                            nullptr, 0)) ? 1 : 0;
}

int tempo_sm100_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                          int ldb, int ldc, void* ws, size_t ws_bytes, void* stream) {
  return tempo::gen::launch(fp16_params(A, B, C, M, N, K, lda, ldb, ldc, ws, ws_bytes),
                            static_cast<cudaStream_t>(stream));
}

int tempo_sm100_gemm_w8a16_applicable(const void* A, const void* W, const void* scale,
                                      const void* zero, const void* C, int M, int N, int K,
                                      int lda, int ldw, int ldc, int quant_kind, int group_size) {
  return tempo::gen::applicable(w8_params(A, W, scale, zero, const_cast<void*>(C), M, N, K, lda,
                                          ldw, ldc, quant_kind, group_size, nullptr, 0)) ? 1 : 0;
}

int tempo_sm100_gemm_w8a16(const void* A, const void* W, const void* scale, const void* zero,
                           void* C, int M, int N, int K, int lda, int ldw, int ldc, int quant_kind,
                           int group_size, void* ws, size_t ws_bytes, void* stream) {
  return tempo::gen::launch(w8_params(A, W, scale, zero, C, M, N, K, lda, ldw, ldc, quant_kind,
                                      group_size, ws, ws_bytes),
                            static_cast<cudaStream_t>(stream));
}

size_t tempo_sm100_workspace_bytes(int M, int N, int K, int weight_kind) {
  tempo::gen::Choice c{};
  cudaError_t e;
  if (weight_kind == 0)
    e = tempo::gen::plan(fp16_params(nullptr, nullptr, nullptr, M, N, K, K, K, N, nullptr,
                                     kPlanAnyWorkspace), &c);
  else
    e = tempo::gen::plan(w8_params(nullptr, nullptr, nullptr, nullptr, nullptr, M, N, K, K,
                                   (K + 15) / 16 * 16, N, weight_kind, 64, nullptr,
                                   kPlanAnyWorkspace), &c);
  return e == cudaSuccess ? c.ws_bytes : 0;
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
  if (swap) return cudaErrorInvalidConfiguration;
  if (weight_kind == 0) {
    if (!fp16_applicable(A, W, C, M, N, K, lda, ldw, ldc)) return cudaErrorInvalidConfiguration;
  } else if (!w8_applicable(A, W, scale, zero, C, M, N, K, lda, ldw, ldc, weight_kind,
                            group_size)) {
    return cudaErrorInvalidConfiguration;
  }
  Hyper h{bn, 0, splits > 1 ? 2 : 1, group_m < 1 ? 1 : group_m, max_ctas};
  h.cta_group = 2;
  Problem pr{weight_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  return run(pr, h, static_cast<cudaStream_t>(stream));
}

int tempo_sm100_pair_resources(int bn, int* out6) { return pair_resources(bn, out6); }

int tempo_sm100_select(int weight_kind, int M, int N, int K, size_t ws_bytes, int* out5) {
  tempo::gen::Choice c{};
  const cudaError_t e =
      weight_kind == 0
          ? tempo::gen::plan(fp16_params(nullptr, nullptr, nullptr, M, N, K, K, K, N, nullptr,
                                         ws_bytes), &c)
          : tempo::gen::plan(w8_params(nullptr, nullptr, nullptr, nullptr, nullptr, M, N, K, K,
                                       (K + 15) / 16 * 16, N, weight_kind, 64, nullptr,
                                       ws_bytes), &c);
  if (e != cudaSuccess) return e;
  if (out5) {
    out5[0] = c.bn;
    out5[1] = c.swap;
    out5[2] = c.splits;
    out5[3] = c.group_m;
    out5[4] = c.stages;
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
  if (M < kExpandMinM || N % 128 || !ws || ws_bytes < kExpandOffset + expand_ws_bytes(N, K))
    return cudaErrorInvalidConfiguration;
  if (!aligned16(ws)) return cudaErrorInvalidValue;
  if (!w8_applicable(A, W, scale, zero, C, M, N, K, lda, ldw, N, quant_kind, group_size) ||
      ldc < N / 2 || (ldc % 8))
    return cudaErrorInvalidConfiguration;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Problem pw{quant_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  // the copy after the counter prefix, which stays as the workspace's other users left it
  __half* wf = reinterpret_cast<__half*>(static_cast<char*>(ws) + kExpandOffset);
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
                   static_cast<__half*>(dst), n, cap, ps, tp, rank, (uint32_t)epoch, wait_ns,
                   static_cast<uint32_t*>(nullptr));
}

int tempo_sm100_allreduce_oneshot_dev(const void* src, void* dst, long long n, long long cap,
                                      void* const* recv, void* const* flags, int tp, int rank,
                                      void* epoch_ctr, int ctas, void* stream) {
  if (!src || !dst || !recv || !flags || !epoch_ctr || tp < 1 || tp > kArMaxTp || rank < 0 ||
      rank >= tp)
    return cudaErrorInvalidValue;
  if (n <= 0 || (n % 8) || n > cap || (cap % 8) || ctas < 1 || ctas > kArMaxCtas)
    return cudaErrorInvalidValue;
  if (!aligned16(src) || !aligned16(dst) || (reinterpret_cast<uintptr_t>(epoch_ctr) & 7u))
    return cudaErrorInvalidValue;
  PeerSet ps{};
  for (int p = 0; p < tp; ++p) {
    if (!recv[p] || !flags[p] || !aligned16(recv[p])) return cudaErrorInvalidValue;
    ps.recv[p] = static_cast<__half*>(recv[p]);
    ps.flags[p] = static_cast<uint32_t*>(flags[p]);
  }
  return launch_ex(k_allreduce_oneshot, dim3(ctas), dim3(256), 0,
                   static_cast<cudaStream_t>(stream), 1, static_cast<const __half*>(src),
                   static_cast<__half*>(dst), n, cap, ps, tp, rank, 0u, kWaitLimitNs,
                   static_cast<uint32_t*>(epoch_ctr));
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
  if (!tempo::gen::applicable(fp16_params(A, B, C, M, N, K, lda, ldb, ldc, nullptr, 0)))
    return cudaErrorInvalidConfiguration;
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
  tempo::gen::Choice c{};
  e = tempo::gen::plan(fp16_params(A, B, C, M, N, K, lda, ldb, ldc, nullptr, kPlanAnyWorkspace),
                       &c);
  if (e != cudaSuccess) return e;
  const size_t need = c.ws_bytes, zero_bytes = c.zero_bytes;
  if (need > (size_t)TEMPO_SM100_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  Hyper h{c.bn, c.swap, c.splits, c.group_m, 0};
  h.cta_group = c.cta_group;
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
