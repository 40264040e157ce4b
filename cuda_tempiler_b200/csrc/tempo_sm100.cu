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

#include "gemm_sm100.cuh"
#include "naive_gemm.cuh"
#include "tempo_sm100.h"

namespace tempo_sm100 {


namespace {

constexpr int kMaxDevices = 64;

// ------------------------------------------------------------------------------------------
// Driver entry point for cuTensorMapEncodeTiled (no -lcuda link dependency).
// ------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major tensor [outer][inner] with row stride `ld` elements; box [box_outer][box_inner].
bool make_map(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int esize, uint64_t inner,
              uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {ld * (uint64_t)esize};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DevInfo {
  int sms = 0;
};

DevInfo dev_info(int dev) {
  static DevInfo info[kMaxDevices];
  static std::once_flag once[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return DevInfo{};
  std::call_once(once[dev], [dev] {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    info[dev].sms = v;
  });
  return info[dev];
}

struct Problem {
  int wkind;  // 0 fp16, 1 int8 per-channel, 2 uint8 group
  const void* A;
  const void* W;
  const void* scale;
  const void* zero;
  void* C;
  int M, N, K;
  long long lda, ldw, ldc;
  int group;
  void* ws;
  size_t ws_bytes;
};

struct Hyper {
  int bn, swap, splits, group_m, max_ctas;
};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t counters_bytes(int tiles) { return ((size_t)tiles * sizeof(int) + 255) / 256 * 256; }

size_t ws_needed(int tiles, int splits, int bn) {
  if (splits <= 1) return 0;
  return counters_bytes(tiles) + (size_t)tiles * splits * 128 * bn * sizeof(float);
}

// ------------------------------------------------------------------------------------------
// Instantiation table.
// ------------------------------------------------------------------------------------------
template <int BN, int WQ, bool SWAP>
cudaError_t launch_inst(const Problem& pr, const Hyper& h, cudaStream_t st) {
  using Cfg = SkelCfg<BN, WQ, SWAP>;
  auto kern = k_gemm_sm100<BN, WQ, SWAP>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    // cudaFuncSetAttribute once per instantiation and device (the reference calls it on every
    // launch, launch.cuh:44-48; it is idempotent but not free).
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr_err[kMaxDevices];
    if (dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [&] {
      attr_err[dev] =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    });
    if (attr_err[dev] != cudaSuccess) return attr_err[dev];
  }
  const int rows_p = SWAP ? pr.N : pr.M;
  const int rows_q = SWAP ? pr.M : pr.N;
  GemmArgs a{};
  a.rows_p = rows_p;
  a.rows_q = rows_q;
  a.K = pr.K;
  a.tiles_p = (rows_p + Cfg::BM - 1) / Cfg::BM;
  a.tiles_q = (rows_q + BN - 1) / BN;
  a.num_kb = (pr.K + Cfg::BK - 1) / Cfg::BK;
  a.splits = std::max(1, std::min(h.splits, a.num_kb));
  const int tiles = a.tiles_p * a.tiles_q;
  a.num_units = tiles * a.splits;
  a.group_m = std::max(1, h.group_m);
  a.C = static_cast<__half*>(pr.C);
  a.ldc = pr.ldc;
  if (a.splits > 1) {
    if (!pr.ws || pr.ws_bytes < ws_needed(tiles, a.splits, BN)) return cudaErrorInvalidValue;
    a.counters = static_cast<int*>(pr.ws);
    a.ws = reinterpret_cast<float*>(static_cast<char*>(pr.ws) + counters_bytes(tiles));
  }
  a.scale = static_cast<const __half*>(pr.scale);
  a.zero = static_cast<const uint8_t*>(pr.zero);
  a.group_size = pr.group > 0 ? pr.group : 1;
  a.groups_per_row = pr.group > 0 ? pr.K / pr.group : 1;
  a.weight_rows = pr.N;

  CUtensorMap mP, mQ, mW, mC;
  std::memset(&mP, 0, sizeof(mP));
  std::memset(&mQ, 0, sizeof(mQ));
  std::memset(&mW, 0, sizeof(mW));
  std::memset(&mC, 0, sizeof(mC));
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const auto SW128 = CU_TENSOR_MAP_SWIZZLE_128B;
  bool ok = true;
  if (SWAP) {
    if (WQ == 0)
      ok &= make_map(&mP, pr.W, F16, 2, pr.K, pr.N, pr.ldw, 64, 128, SW128);
    else
      ok &= make_map(&mW, pr.W, U8, 1, pr.K, pr.N, pr.ldw, 64, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    ok &= make_map(&mQ, pr.A, F16, 2, pr.K, pr.M, pr.lda, 64, BN, SW128);
  } else {
    ok &= make_map(&mP, pr.A, F16, 2, pr.K, pr.M, pr.lda, 64, 128, SW128);
    if (WQ == 0)
      ok &= make_map(&mQ, pr.W, F16, 2, pr.K, pr.N, pr.ldw, 64, BN, SW128);
    else
      ok &= make_map(&mW, pr.W, U8, 1, pr.K, pr.N, pr.ldw, 64, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    ok &= make_map(&mC, pr.C, F16, 2, pr.N, pr.M, pr.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (!ok) return cudaErrorInvalidValue;

  const int sms = dev_info(dev).sms;
  int grid = std::min(a.num_units, h.max_ctas > 0 ? h.max_ctas : sms);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, st>>>(mP, mQ, mW, mC, a);
  return cudaGetLastError();
}

using LaunchFn = cudaError_t (*)(const Problem&, const Hyper&, cudaStream_t);

struct InstEntry {
  int wkind, bn, swap;
  LaunchFn fn;
  const void* kern;
  int threads, smem, stages, tmem_cols;
};

#define TEMPO_INST(BN, WQ, SWAP)                                                        \
  InstEntry {                                                                           \
    WQ, BN, SWAP, &launch_inst<BN, WQ, SWAP>,                                           \
        reinterpret_cast<const void*>(&k_gemm_sm100<BN, WQ, SWAP>),                     \
        SkelCfg<BN, WQ, SWAP>::THREADS, SkelCfg<BN, WQ, SWAP>::SMEM,                    \
        SkelCfg<BN, WQ, SWAP>::STAGES, SkelCfg<BN, WQ, SWAP>::TMEM_COLS                 \
  }
#define TEMPO_INST_WQ(BN, SWAP) TEMPO_INST(BN, 0, SWAP), TEMPO_INST(BN, 1, SWAP), TEMPO_INST(BN, 2, SWAP)

const InstEntry kInst[] = {
    TEMPO_INST_WQ(16, true),  TEMPO_INST_WQ(32, true),   TEMPO_INST_WQ(64, true),
    TEMPO_INST_WQ(128, true), TEMPO_INST_WQ(64, false),  TEMPO_INST_WQ(128, false),
    TEMPO_INST_WQ(256, false),
};

const InstEntry* find_inst(int wkind, int bn, int swap) {
  for (const auto& e : kInst)
    if (e.wkind == wkind && e.bn == bn && e.swap == (swap ? 1 : 0)) return &e;
  return nullptr;
}

// ------------------------------------------------------------------------------------------
// The M-ladder (generated from select.py into dispatch.inc) and the split-K cost model.
// ------------------------------------------------------------------------------------------
struct LadderRow {
  int m_max;  // inclusive upper bound on M (0x7fffffff = everything else)
  int bn, swap, group_m;
};

#include "dispatch.inc"

const LadderRow* ladder_row(int wkind, int M) {
  const LadderRow* rows = wkind == 0 ? kLadderFp16 : kLadderW8;
  const int n = wkind == 0 ? (int)(sizeof(kLadderFp16) / sizeof(LadderRow))
                           : (int)(sizeof(kLadderW8) / sizeof(LadderRow));
  for (int i = 0; i < n; ++i)
    if (M <= rows[i].m_max) return &rows[i];
  return nullptr;
}

// Time model in units of one k-block of one tile: waves * (k-blocks per unit + fill), plus a
// fix-up charge per extra split.  Picks the k-split that best fills `sms` persistent CTAs.
int choose_splits(int tiles, int num_kb, int sms, int bn, size_t ws_bytes) {
  if (sms <= 0) return 1;
  auto cost = [&](int s) {
    const long long units = (long long)tiles * s;
    const long long waves = (units + sms - 1) / sms;
    const long long per = (num_kb + s - 1) / s;
    return (double)waves * (double)(per + 4) + (s > 1 ? 2.0 + 0.25 * s : 0.0);
  };
  int best = 1;
  double best_c = cost(1);
  const int smax = std::min(32, num_kb / 2);
  for (int s = 2; s <= smax; ++s) {
    if (ws_needed(tiles, s, bn) > ws_bytes) break;
    const double c = cost(s);
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
  const int rows_p = h.swap ? N : M, rows_q = h.swap ? M : N;
  const int tiles = ((rows_p + 127) / 128) * ((rows_q + h.bn - 1) / h.bn);
  const int num_kb = (K + 63) / 64;
  h.splits = choose_splits(tiles, num_kb, sms, h.bn, ws_bytes);
  return find_inst(wkind, h.bn, h.swap) != nullptr;
}

bool fp16_applicable(const void* A, const void* B, const void* C, int M, int N, int K, long long lda,
                     long long ldb, long long ldc) {
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (!A || !B || !C) return false;
  if ((K % 8) || (N % 8)) return false;
  if (lda < K || ldb < K || ldc < N) return false;
  if ((lda % 8) || (ldb % 8) || (ldc % 8)) return false;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C)) return false;
  return true;
}

bool w8_applicable(const void* A, const void* W, const void* scale, const void* zero, const void* C,
                   int M, int N, int K, long long lda, long long ldw, long long ldc, int kind,
                   int group) {
  if (kind != TEMPO_W8_INT8_PER_CHANNEL && kind != TEMPO_W8_UINT8_GROUP) return false;
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (!A || !W || !C || !scale) return false;
  if ((K % 16) || (N % 8)) return false;
  if (lda < K || ldw < K || ldc < N) return false;
  if ((lda % 8) || (ldw % 16) || (ldc % 8)) return false;
  if (!aligned16(A) || !aligned16(W) || !aligned16(C)) return false;
  if (kind == TEMPO_W8_UINT8_GROUP) {
    if (!zero || group <= 0 || (group % 64) || (K % group)) return false;
  }
  return true;
}

cudaError_t run(const Problem& pr, const Hyper& h, cudaStream_t st) {
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
  Hyper h{};
  if (!select_hyper(quant_kind, M, N, K, ws ? ws_bytes : 0, h, current_sms()))
    return cudaErrorInvalidConfiguration;
  Problem pr{quant_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  return run(pr, h, static_cast<cudaStream_t>(stream));
}

size_t tempo_sm100_workspace_bytes(int M, int N, int K, int weight_kind) {
  Hyper h{};
  if (!select_hyper(weight_kind, M, N, K, (size_t)1 << 40, h, current_sms())) return 0;
  const int rows_p = h.swap ? N : M, rows_q = h.swap ? M : N;
  const int tiles = ((rows_p + 127) / 128) * ((rows_q + h.bn - 1) / h.bn);
  return ws_needed(tiles, h.splits, h.bn);
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
  Hyper h{bn, swap ? 1 : 0, splits < 1 ? 1 : splits, group_m < 1 ? 1 : group_m, max_ctas};
  Problem pr{weight_kind, A, W, scale, zero, C, M, N, K, lda, ldw, ldc, group_size, ws, ws_bytes};
  return run(pr, h, static_cast<cudaStream_t>(stream));
}

int tempo_sm100_select(int weight_kind, int M, int N, int K, size_t ws_bytes, int* out5) {
  Hyper h{};
  if (!select_hyper(weight_kind, M, N, K, ws_bytes, h, current_sms()))
    return cudaErrorInvalidConfiguration;
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
  if (!select_hyper(0, M, N, K, (size_t)1 << 40, h, current_sms()))
    return cudaErrorInvalidConfiguration;
  const int rows_p = h.swap ? N : M, rows_q = h.swap ? M : N;
  const int tiles = ((rows_p + 127) / 128) * ((rows_q + h.bn - 1) / h.bn);
  const size_t need = ws_needed(tiles, h.splits, h.bn);
  if (need > (size_t)TEMPO_SM100_NOALLOC_SCRATCH_BYTES) return cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (need > 0) {
    // The counters must start at zero; the array keeps whatever the previous call left.
    e = cudaMemsetAsync(scratch, 0, counters_bytes(tiles), st);
    if (e != cudaSuccess) return e;
  }
  Problem pr{0, A, B, nullptr, nullptr, C, M, N, K, lda, ldb, ldc, 0, scratch,
             (size_t)TEMPO_SM100_NOALLOC_SCRATCH_BYTES};
  return run(pr, h, st);
}
