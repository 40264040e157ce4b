// launch.cuh -- host layer of the sm_100a GEMM skeleton family: TMA descriptor construction,
// the instantiation table (one entry per (BN, weight kind, swap) hyperform family member), the
// persistent-grid and 2-CTA launches, the work planners and the ladder-row dispatcher engine.
// Everything here has internal linkage: the ship stage freezes it into the first half of each
// shipped launch.cu (the single translation unit that instantiates the kernels, as the
// reference's kernels/shipped/gemm_fp16/sm_70/launch.cu is); the public POD ABI is the
// separate shipped launch.cuh.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <mutex>

#include "kernel.cuh"
#include "naive.cuh"

#ifndef TEMPO_W8_INT8_PER_CHANNEL
#define TEMPO_W8_INT8_PER_CHANNEL 1
#define TEMPO_W8_UINT8_GROUP 2
#endif

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
// Encoding a descriptor costs about a microsecond of host time, several per launch, so the
// descriptors of recent calls are kept in a small per-thread cache keyed by every argument (a
// descriptor holds only the address and the geometry, so a hit is exact whatever the memory
// holds now).
struct MapKey {
  const void* ptr;
  uint64_t inner, outer, ld;
  uint32_t box_inner, box_outer;
  int dt, esize, sw;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && inner == o.inner && outer == o.outer && ld == o.ld &&
           box_inner == o.box_inner && box_outer == o.box_outer && dt == o.dt &&
           esize == o.esize && sw == o.sw;
  }
};

struct MapSlot {
  MapKey key;
  CUtensorMap map;
  bool used = false;
};

constexpr int kMapCacheSlots = 256;

bool make_map(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int esize, uint64_t inner,
              uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle sw) {
  const MapKey key{ptr, inner, outer, ld, box_inner, box_outer, (int)dt, esize, (int)sw};
  uint64_t h = reinterpret_cast<uintptr_t>(ptr) * 0x9E3779B97F4A7C15ull;
  for (uint64_t v : {inner, outer, ld, (uint64_t)box_inner << 32 | box_outer,
                     (uint64_t)dt << 40 | (uint64_t)esize << 20 | (uint64_t)sw})
    h = (h ^ v) * 0x100000001B3ull;
  thread_local MapSlot cache[kMapCacheSlots];
  MapSlot& slot = cache[(h >> 24) % kMapCacheSlots];
  if (slot.used && slot.key == key) {
    *m = slot.map;
    return true;
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {ld * (uint64_t)esize};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  if (fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  slot.key = key;
  slot.map = *m;
  slot.used = true;
  return true;
}

// Launch attributes every product kernel gets: programmatic dependent launch (the kernel
// waits for its predecessors in the stream with griddepcontrol.wait after a prologue that
// touches no shared global memory), and a cluster shape when cluster_x > 1.  Setting
// TEMPO_SM100_PDL=0 in the environment turns programmatic launch off.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("TEMPO_SM100_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t st, int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
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
  void* ws;         // workspace: the arrival-counter prefix at its start
  size_t ws_bytes;  // bytes of it for counters + fp32 partials
  // where the fp32 partials start; nullptr: right after the counter prefix.  The W8A16
  // prefill puts its expanded weights between the two, so that nothing but counters ever
  // occupies the prefix of a workspace a caller reuses across problems.
  void* ws_parts = nullptr;
};

struct Hyper {
  int bn, swap, splits, group_m, max_ctas;
  int cta_group = 1;  // 2: 256 x BN tiles on a 2-CTA cluster (fp16 prefill only)
};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Split workspace layout, the same for every problem: a fixed prefix of kMaxCounters arrival
// counters, then the fp32 partials.  A fixed prefix keeps one problem's counters off another
// problem's leftover partials when a caller reuses one workspace for different shapes; every
// launch leaves the counters it used at zero.
constexpr int kMaxCounters = 16384;
constexpr size_t kCounterBytes = (size_t)kMaxCounters * sizeof(int);  // 64 KiB

// Bytes of the counter prefix that n counters occupy (what must be zero before a launch).
size_t counters_used_bytes(int n) { return ((size_t)n * sizeof(int) + 255) / 256 * 256; }

// k-splits up to this count run inside one cluster and reduce through distributed shared
// memory (no workspace); larger counts go through the global workspace.
constexpr int kMaxClusterSplit = kMaxClusterSplitDev;

size_t ws_needed(int tiles, int splits, int bn) {
  if (splits <= kMaxClusterSplit) return 0;
  if (tiles > kMaxCounters) return ~(size_t)0;
  return kCounterBytes + (size_t)tiles * splits * 128 * bn * sizeof(float);
}

// ------------------------------------------------------------------------------------------
// Instantiation table.
// ------------------------------------------------------------------------------------------
template <int BN, int WQ, bool SWAP, bool SMEMDQ = false>
cudaError_t launch_inst(const Problem& pr, const Hyper& h, cudaStream_t st) {
  using Cfg = SkelCfg<BN, WQ, SWAP, SMEMDQ>;
  auto kern = k_gemm_sm100<BN, WQ, SWAP, SMEMDQ>;
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
  a.num_kb = (pr.K + Cfg::KS - 1) / Cfg::KS;
  a.splits = std::max(1, std::min(h.splits, a.num_kb));
  const int tiles = a.tiles_p * a.tiles_q;
  a.num_units = tiles * a.splits;
  a.group_m = std::max(1, h.group_m);
  a.C = static_cast<__half*>(pr.C);
  a.ldc = pr.ldc;
  a.cluster_split = (a.splits > 1 && a.splits <= kMaxClusterSplit) ? a.splits : 0;
  if (a.splits > kMaxClusterSplit) {
    if (!pr.ws || pr.ws_bytes < ws_needed(tiles, a.splits, BN)) return cudaErrorInvalidValue;
    a.counters = static_cast<int*>(pr.ws);
    a.ws = reinterpret_cast<float*>(pr.ws_parts ? static_cast<char*>(pr.ws_parts)
                                                : static_cast<char*>(pr.ws) + kCounterBytes);
  }
  a.scale = static_cast<const __half*>(pr.scale);
  a.zero = static_cast<const uint8_t*>(pr.zero);
  a.group_size = pr.group > 0 ? pr.group : 1;
  a.groups_per_row = pr.group > 0 ? pr.K / pr.group : 1;
  a.weight_rows = pr.N;

  CUtensorMap mP, mQ, mW, mC, mS, mZ;
  std::memset(&mS, 0, sizeof(mS));
  std::memset(&mZ, 0, sizeof(mZ));
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
    else if (Cfg::TA)
      // one 128-byte row per weight row and request; the 128-byte swizzle keeps the dequant
      // threads' per-row reads bank-conflict free
      ok &= make_map(&mW, pr.W, U8, 1, pr.K, pr.N, pr.ldw, Cfg::KS, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    else  // shared-memory dequant: 64-byte raw rows, as the non-swapped W8A16 tiles read them
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
  if (WQ == 2) {
    // group-wise scale fp16 [K/G][N] and zero uint8 [K/G][N]: one row segment per k-block
    const int wrows = SWAP ? Cfg::BM : BN;
    const uint64_t groups = (uint64_t)(pr.K / pr.group);
    const int grows = std::max(1, Cfg::KS / pr.group);  // group rows one stage spans
    ok &= make_map(&mS, pr.scale, F16, 2, pr.N, groups, pr.N, wrows, grows, CU_TENSOR_MAP_SWIZZLE_NONE);
    ok &= make_map(&mZ, pr.zero, U8, 1, pr.N, groups, pr.N, wrows, grows, CU_TENSOR_MAP_SWIZZLE_NONE);
    a.sz_bytes = wrows * 3 * grows;
  }
  if (!ok) return cudaErrorInvalidValue;

  if (a.cluster_split > 1)  // one CTA per unit, the k-slices of a tile in one cluster
    return launch_ex(kern, dim3(a.num_units), dim3(Cfg::THREADS), Cfg::SMEM, st, a.splits, mP,
                     mQ, mW, mC, mS, mZ, a);
  const int sms = dev_info(dev).sms;
  int grid = std::min(a.num_units, h.max_ctas > 0 ? h.max_ctas : sms);
  if (grid <= 0) return cudaErrorInvalidConfiguration;
  return launch_ex(kern, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM, st, 1, mP, mQ, mW, mC, mS,
                   mZ, a);
}

// Decode-sized streaming GEMV (hyperform bn == 0): M <= 16, one CTA of kGemvThreads threads
// per R weight rows.
template <int WQ, int MM, int R>
cudaError_t launch_gemv(const Problem& pr, cudaStream_t st) {
  const int grid = (pr.N + R - 1) / R;
  return launch_ex(k_gemv_sm100<WQ, MM, R>, dim3(grid), dim3(kGemvThreads), 0, st, 1,
                   static_cast<const __half*>(pr.A), static_cast<const uint8_t*>(pr.W),
                   static_cast<const __half*>(pr.scale), static_cast<const uint8_t*>(pr.zero),
                   static_cast<__half*>(pr.C), pr.M, pr.N, pr.K, (long long)pr.lda,
                   (long long)pr.ldw, (long long)pr.ldc, pr.group > 0 ? pr.group : 1);
}

// Rows per CTA: the widest R in {4, 2, 1} that still gives at least kGemvMinCtasPerSm CTAs
// per SM (so the block scheduler can balance the bytes each SM streams); wider R reuses each
// activation chunk over more weight rows.  8 and 16 activation rows keep R <= 2 so the
// accumulators stay in registers.
constexpr int kGemvMinCtasPerSm = 12;

int gemv_rows(int N, int M, int sms) {
  const long long want = (long long)kGemvMinCtasPerSm * (sms > 0 ? sms : 148);
  const int rmax = M > 4 ? 2 : 4;
  for (int r = rmax; r > 1; r >>= 1)
    if ((long long)N / r >= want) return r;
  return 1;
}

template <int WQ, int R>
cudaError_t gemv_by_m(const Problem& pr, cudaStream_t st) {
  if (pr.M == 1) return launch_gemv<WQ, 1, R>(pr, st);
  if (pr.M == 2) return launch_gemv<WQ, 2, R>(pr, st);
  if (pr.M <= 4) return launch_gemv<WQ, 4, R>(pr, st);
  if (R <= 2) {
    if (pr.M <= 8) return launch_gemv<WQ, 8, (R <= 2 ? R : 2)>(pr, st);
    return launch_gemv<WQ, 16, (R <= 2 ? R : 2)>(pr, st);
  }
  return cudaErrorInvalidConfiguration;
}

template <int WQ>
cudaError_t gemv_by_rows(const Problem& pr, int rows, cudaStream_t st) {
  if (rows == 4) return gemv_by_m<WQ, 4>(pr, st);
  if (rows == 2) return gemv_by_m<WQ, 2>(pr, st);
  return gemv_by_m<WQ, 1>(pr, st);
}

// The tensor-core decode GEMV (k_gemv_mma_sm100): 16 weight rows per CTA, k split over a
// cluster of `splits` CTAs -- the smallest power of two (at most 8) that gives every SM at
// least kGemvMmaMinCtasPerSm CTAs.
constexpr int kGemvMmaMinCtasPerSm = 8;

int gemv_mma_splits(int N, int K, int wkind, int sms) {
  const long long groups = (N + 15) / 16;
  const long long want = (long long)kGemvMmaMinCtasPerSm * (sms > 0 ? sms : 148);
  const int nch = K / (wkind == 0 ? 8 : 16);
  int s = 1;
  while (s < kGemvMmaMaxSplit && groups * s < want && nch / (2 * s) >= 16) s *= 2;
  return s;
}

template <int WQ, int MG>
cudaError_t launch_gemv_mma(const Problem& pr, int splits, cudaStream_t st) {
  const int grid = ((pr.N + 15) / 16) * splits;
  return launch_ex(k_gemv_mma_sm100<WQ, MG>, dim3(grid), dim3(kGemvThreads), 0, st, splits,
                   static_cast<const __half*>(pr.A), static_cast<const uint8_t*>(pr.W),
                   static_cast<const __half*>(pr.scale), static_cast<const uint8_t*>(pr.zero),
                   static_cast<__half*>(pr.C), pr.M, pr.N, pr.K, (long long)pr.lda,
                   (long long)pr.ldw, (long long)pr.ldc, pr.group > 0 ? pr.group : 1, splits);
}

template <int WQ>
cudaError_t gemv_mma_by_m(const Problem& pr, int splits, cudaStream_t st) {
  if (pr.M <= 8) return launch_gemv_mma<WQ, 1>(pr, splits, st);
  return launch_gemv_mma<WQ, 2>(pr, splits, st);
}

constexpr int kGemvMaxM = 16;
// Activation rows from which the tensor-core GEMV takes over from the CUDA-core one (measured
// on the BASELINE shapes: fp16 weights from 5 rows, 8-bit weights -- whose CUDA-core dequant
// adds to the FMA issue -- from 3).
int gemv_mma_min_m(int wkind) { return wkind == 0 ? 5 : 3; }

// variant (a GEMV hyperform's group_m): 1 = CUDA-core, 2 = tensor-core, anything else by M
// (CUDA-core below gemv_mma_min_m, tensor-core from it).
cudaError_t run_gemv(const Problem& pr, cudaStream_t st, int variant = 0) {
  if (pr.M < 1 || pr.M > kGemvMaxM) return cudaErrorInvalidConfiguration;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = dev_info(dev).sms;
  const bool mma = variant == 2 || (variant != 1 && pr.M >= gemv_mma_min_m(pr.wkind));
  if (mma) {
    const int splits = gemv_mma_splits(pr.N, pr.K, pr.wkind, sms);
    switch (pr.wkind) {
      case 0: return gemv_mma_by_m<0>(pr, splits, st);
      case 1: return gemv_mma_by_m<1>(pr, splits, st);
      case 2: return gemv_mma_by_m<2>(pr, splits, st);
      default: return cudaErrorInvalidConfiguration;
    }
  }
  const int rows = gemv_rows(pr.N, pr.M, sms);
  switch (pr.wkind) {
    case 0: return gemv_by_rows<0>(pr, rows, st);
    case 1: return gemv_by_rows<1>(pr, rows, st);
    case 2: return gemv_by_rows<2>(pr, rows, st);
    default: return cudaErrorInvalidConfiguration;
  }
}

// W8A16 at prefill-sized M: expand the 8-bit weights to fp16 in the workspace, then the fp16
// dispatch (2-CTA tiles) runs on the copy.  kExpandMinM and the workspace decide.
constexpr int kExpandMinM = 512;

size_t expand_ws_bytes(int N, int K) { return ((size_t)N * K * 2 + 255) / 256 * 256; }

// The expanded weights sit right after the counter prefix of the workspace (never at its
// start: a workspace reused by a later split-K launch must still hold zeroed counters there).
constexpr size_t kExpandOffset = kCounterBytes;

// Rows [n0, n0 + rows) of the weights expanded into out (rows x K, dense); wait as in
// k_expand_w8.
cudaError_t launch_expand_rows(const Problem& pr, int n0, int rows, __half* out, bool wait,
                               cudaStream_t st) {
  const long long n = (long long)rows * (pr.K / 16);
  const unsigned grid = (unsigned)((n + 255) / 256);
  const uint8_t* W = static_cast<const uint8_t*>(pr.W) + (long long)n0 * pr.ldw;
  const __half* sc = static_cast<const __half*>(pr.scale) + n0;
  const uint8_t* z = pr.zero ? static_cast<const uint8_t*>(pr.zero) + n0 : nullptr;
  const int g = pr.group > 0 ? pr.group : 16;
  if (pr.wkind == kWInt8PerChannel)
    return launch_ex(k_expand_w8<kWInt8PerChannel>, dim3(grid), dim3(256), 0, st, 1, W, sc, z,
                     out, rows, pr.K, (long long)pr.ldw, g, pr.N, wait ? 1 : 0);
  if (pr.wkind == kWUint8Group)
    return launch_ex(k_expand_w8<kWUint8Group>, dim3(grid), dim3(256), 0, st, 1, W, sc, z, out,
                     rows, pr.K, (long long)pr.ldw, g, pr.N, wait ? 1 : 0);
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_expand(const Problem& pr, __half* out, cudaStream_t st) {
  return launch_expand_rows(pr, 0, pr.N, out, true, st);
}

using LaunchFn = cudaError_t (*)(const Problem&, const Hyper&, cudaStream_t);

struct InstEntry {
  int wkind, bn, swap;
  LaunchFn fn;
  const void* kern;
  int threads, smem, stages, tmem_cols;
};

// swap code in the table: 0 = not swapped, 1 = swapped (8-bit weights dequantised into TMEM),
// 2 = swapped with the 8-bit weights dequantised into shared memory
#define TEMPO_INST4(BN, WQ, SWAP, DQ, CODE)                                             \
  InstEntry {                                                                           \
    WQ, BN, CODE, &launch_inst<BN, WQ, SWAP, DQ>,                                       \
        reinterpret_cast<const void*>(&k_gemm_sm100<BN, WQ, SWAP, DQ>),                 \
        SkelCfg<BN, WQ, SWAP, DQ>::THREADS, SkelCfg<BN, WQ, SWAP, DQ>::SMEM,            \
        SkelCfg<BN, WQ, SWAP, DQ>::STAGES, SkelCfg<BN, WQ, SWAP, DQ>::TMEM_COLS         \
  }
#define TEMPO_INST(BN, WQ, SWAP) TEMPO_INST4(BN, WQ, SWAP, false, SWAP ? 1 : 0)
#define TEMPO_INST_WQ(BN, SWAP) TEMPO_INST(BN, 0, SWAP), TEMPO_INST(BN, 1, SWAP), TEMPO_INST(BN, 2, SWAP)
#define TEMPO_INST_SDQ(BN) TEMPO_INST4(BN, 1, true, true, 2), TEMPO_INST4(BN, 2, true, true, 2)

const InstEntry kInst[] = {
    TEMPO_INST_WQ(16, true),  TEMPO_INST_WQ(32, true),   TEMPO_INST_WQ(64, true),
    TEMPO_INST_WQ(128, true), TEMPO_INST_WQ(64, false),  TEMPO_INST_WQ(128, false),
    TEMPO_INST_WQ(256, false),
    TEMPO_INST_SDQ(32),       TEMPO_INST_SDQ(64),        TEMPO_INST_SDQ(128),
};

// Work split of the 2-CTA kernel.  P clusters (one per SM pair) take whole 256 x BN tiles in
// turn.  When the tiles leave a ragged last wave, the tiles of that wave (or every tile, with
// fewer tiles than two waves) can instead run as a split tail: each cut into S k-slices, the
// slices numbered k-slice major so concurrent clusters read neighbouring k ranges, and the
// tile's last slice to finish adds the fp32 partials up in k order.  Cost in tile times:
// whole waves + ceil(R * S / P) / S + S x (a slice's fixup against the tile's MMA cycles); the
// tail is taken when it saves at least 3 %.  Workspace: the counter prefix (2 per tail tile), then R * S slots of
// 2 x [BN][128] fp32.
struct PairPlan {
  int clusters = 0, tiles = 0, num_kb = 0;
  int sk_tile0 = 0, sk_tiles = 0, sk_splits = 0;
  size_t ws_bytes = 0;  // workspace the tail needs (0: none)
  double cost = 0;      // modelled time in tile times
};

constexpr int kPairMinSlice = 4;  // fewest k-blocks in one tail k-slice
constexpr double kPairSliceFixCycles = 20000.0;  // cost of one tail k-slice's fp32 round trip

PairPlan pair_plan(int M, int N, int K, int bn, int sms, int max_ctas, bool split_tail,
                   size_t ws_bytes) {
  PairPlan pl;
  pl.tiles = ((M + 255) / 256) * ((N + bn - 1) / bn);
  pl.num_kb = (K + 63) / 64;
  const int P = std::max(1, (max_ctas > 0 ? std::min(max_ctas, sms) : sms) / 2);
  pl.clusters = std::min(pl.tiles, P);
  pl.sk_tile0 = pl.tiles;
  pl.cost = (double)((pl.tiles + P - 1) / P);
  if (!split_tail || pl.tiles % P == 0) return pl;
  const int R = pl.tiles >= P ? pl.tiles % P : pl.tiles;
  const int full = (pl.tiles - R) / P;
  // a k-slice's partial write and read-back, against a tile's 2 * bn cycles per k-block:
  // ~20000 cycles (measured on B200: down M = 1024 with 3 slices on 18 tail tiles saves 8 %
  // against two whole waves; on the 27B-class shapes at M = 512 every tail lost to whole waves)
  const double fix = kPairSliceFixCycles / (pl.num_kb * 2.0 * bn);
  double best = pl.cost * 0.97;
  int best_s = 0;
  // at most 3 P tail units: 3 waves of slices, and (at bn 256) under 58 MB of partials
  for (int S = 2; S <= 16 && S * kPairMinSlice <= pl.num_kb && R * S <= 3 * P; ++S) {
    const size_t need = kCounterBytes + (size_t)R * S * 2 * 128 * (size_t)bn * sizeof(float);
    if (need > ws_bytes) break;
    const double c = full + (double)((R * S + P - 1) / P) / S + S * fix;
    if (c < best) {
      best = c;
      best_s = S;
    }
  }
  if (best_s == 0) return pl;
  pl.clusters = P;
  pl.sk_tile0 = pl.tiles - R;
  pl.sk_tiles = R;
  pl.sk_splits = best_s;
  pl.ws_bytes = kCounterBytes + (size_t)R * best_s * 2 * 128 * (size_t)bn * sizeof(float);
  pl.cost = best;
  return pl;
}

// 2-CTA (cta_group::2) fp16 prefill launch: persistent clusters of two CTAs; h.splits > 1
// allows the split tail of pair_plan.
template <int BN, bool SWIGLU = false>
cudaError_t launch_pair(const Problem& pr, const Hyper& h, cudaStream_t st) {
  using Cfg = PairCfg<BN>;
  auto kern = k_gemm_sm100_pair<BN, SWIGLU>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr_err[kMaxDevices];
    if (dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [&] {
      attr_err[dev] =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    });
    if (attr_err[dev] != cudaSuccess) return attr_err[dev];
  }
  if (pr.wkind != 0 || h.swap) return cudaErrorInvalidConfiguration;
  if (SWIGLU && (pr.N % 128 || (BN != 128 && BN != 256))) return cudaErrorInvalidConfiguration;
  // the fused SwiGLU epilogue has no split tail (its partial sums would be pre-activation)
  const PairPlan pl = pair_plan(pr.M, pr.N, pr.K, BN, dev_info(dev).sms, h.max_ctas,
                                !SWIGLU && h.splits > 1,
                                pr.ws ? pr.ws_bytes : 0);
  GemmArgs a{};
  a.rows_p = pr.M;
  a.rows_q = pr.N;
  a.K = pr.K;
  a.tiles_p = (pr.M + 255) / 256;
  a.tiles_q = (pr.N + BN - 1) / BN;
  a.num_kb = (pr.K + Cfg::BK - 1) / Cfg::BK;
  a.splits = 1;
  a.num_units = a.tiles_p * a.tiles_q;
  a.group_m = std::max(1, h.group_m / 2);  // raster groups counted in 256-row tiles
  a.C = static_cast<__half*>(pr.C);
  a.ldc = pr.ldc;
  a.weight_rows = pr.N;
  a.sk_tile0 = pl.sk_tile0;
  a.sk_tiles = pl.sk_tiles;
  a.sk_splits = pl.sk_splits;
  if (pl.sk_splits > 0) {
    if (!pr.ws || pr.ws_bytes < pl.ws_bytes) return cudaErrorInvalidValue;
    a.counters = static_cast<int*>(pr.ws);
    a.ws = reinterpret_cast<float*>(pr.ws_parts ? static_cast<char*>(pr.ws_parts)
                                                : static_cast<char*>(pr.ws) + kCounterBytes);
  }
  CUtensorMap mA, mB, mC;
  std::memset(&mA, 0, sizeof(mA));
  std::memset(&mB, 0, sizeof(mB));
  std::memset(&mC, 0, sizeof(mC));
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  bool ok = make_map(&mA, pr.A, F16, 2, pr.K, pr.M, pr.lda, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  ok &= make_map(&mB, pr.W, F16, 2, pr.K, pr.N, pr.ldw, 64, BN / 2, CU_TENSOR_MAP_SWIZZLE_128B);
  ok &= make_map(&mC, pr.C, F16, 2, SWIGLU ? pr.N / 2 : pr.N, pr.M, pr.ldc, 32, 32,
                 CU_TENSOR_MAP_SWIZZLE_64B);
  if (!ok) return cudaErrorInvalidValue;
  return launch_ex(kern, dim3(2 * pl.clusters), dim3(Cfg::THREADS), Cfg::SMEM, st, 2, mA, mB, mC,
                   a);
}

// W8A16 2-CTA launch (k_gemm_sm100_pair_w8): persistent clusters; h.splits > 1 allows the
// split tail of pair_plan (given the workspace it needs).
template <int BN, int WQ>
cudaError_t launch_pair_w8(const Problem& pr, const Hyper& h, cudaStream_t st) {
  using Cfg = PairW8Cfg<BN>;
  auto kern = k_gemm_sm100_pair_w8<BN, WQ>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    static std::once_flag once[kMaxDevices];
    static cudaError_t attr_err[kMaxDevices];
    if (dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [&] {
      attr_err[dev] =
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    });
    if (attr_err[dev] != cudaSuccess) return attr_err[dev];
  }
  if (pr.wkind != WQ || h.swap) return cudaErrorInvalidConfiguration;
  if (WQ == kWUint8Group && (pr.group <= 0 || pr.group % Cfg::BK || pr.K % pr.group || pr.N % 16))
    return cudaErrorInvalidConfiguration;
  const PairPlan pl = pair_plan(pr.M, pr.N, pr.K, BN, dev_info(dev).sms, h.max_ctas,
                                h.splits > 1, pr.ws ? pr.ws_bytes : 0);
  GemmArgs a{};
  a.rows_p = pr.M;
  a.rows_q = pr.N;
  a.K = pr.K;
  a.tiles_p = (pr.M + 255) / 256;
  a.tiles_q = (pr.N + BN - 1) / BN;
  a.num_kb = (pr.K + Cfg::BK - 1) / Cfg::BK;
  a.splits = 1;
  a.num_units = a.tiles_p * a.tiles_q;
  a.group_m = std::max(1, h.group_m / 2);  // raster groups counted in 256-row tiles
  a.C = static_cast<__half*>(pr.C);
  a.ldc = pr.ldc;
  a.weight_rows = pr.N;
  a.scale = static_cast<const __half*>(pr.scale);
  a.zero = static_cast<const uint8_t*>(pr.zero);
  a.group_size = pr.group > 0 ? pr.group : 1;
  a.groups_per_row = pr.group > 0 ? pr.K / pr.group : 1;
  a.sk_tile0 = pl.sk_tile0;
  a.sk_tiles = pl.sk_tiles;
  a.sk_splits = pl.sk_splits;
  if (pl.sk_splits > 0) {
    if (!pr.ws || pr.ws_bytes < pl.ws_bytes) return cudaErrorInvalidValue;
    a.counters = static_cast<int*>(pr.ws);
    a.ws = reinterpret_cast<float*>(pr.ws_parts ? static_cast<char*>(pr.ws_parts)
                                                : static_cast<char*>(pr.ws) + kCounterBytes);
  }
  CUtensorMap mA, mW, mC, mS, mZ;
  std::memset(&mA, 0, sizeof(mA));
  std::memset(&mW, 0, sizeof(mW));
  std::memset(&mC, 0, sizeof(mC));
  std::memset(&mS, 0, sizeof(mS));
  std::memset(&mZ, 0, sizeof(mZ));
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  bool ok = make_map(&mA, pr.A, F16, 2, pr.K, pr.M, pr.lda, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  // raw weights: rows of 64 bytes, unswizzled (the dequant warps apply the MMA's swizzle)
  ok &= make_map(&mW, pr.W, U8, 1, pr.K, pr.N, pr.ldw, 64, BN / 2, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (WQ == kWUint8Group) {
    const int ng = pr.K / pr.group;
    ok &= make_map(&mS, pr.scale, F16, 2, pr.N, ng, pr.N, BN / 2, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    ok &= make_map(&mZ, pr.zero, U8, 1, pr.N, ng, pr.N, BN / 2, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  ok &= make_map(&mC, pr.C, F16, 2, pr.N, pr.M, pr.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!ok) return cudaErrorInvalidValue;
  return launch_ex(kern, dim3(2 * pl.clusters), dim3(Cfg::THREADS), Cfg::SMEM, st, 2, mA, mW, mC,
                   mS, mZ, a);
}

cudaError_t run_pair(const Problem& pr, const Hyper& h, cudaStream_t st) {
  switch (h.bn) {
    case 256: return launch_pair<256>(pr, h, st);
    case 224: return launch_pair<224>(pr, h, st);
    case 192: return launch_pair<192>(pr, h, st);
    case 160: return launch_pair<160>(pr, h, st);
    case 128: return launch_pair<128>(pr, h, st);
    default: return cudaErrorInvalidConfiguration;
  }
}

// 2-CTA W8A16 tiles (8-bit weights dequantised in shared memory by 8 warps per CTA).
constexpr int kPairW8Bn[] = {256, 128};
constexpr double kPairW8Eff[] = {1.0, 0.55};

cudaError_t run_pair_w8(const Problem& pr, const Hyper& h, cudaStream_t st) {
  const bool pc = pr.wkind == kWInt8PerChannel;
  if (!pc && pr.wkind != kWUint8Group) return cudaErrorInvalidConfiguration;
  switch (h.bn) {
    case 256: return pc ? launch_pair_w8<256, 1>(pr, h, st) : launch_pair_w8<256, 2>(pr, h, st);
    case 128: return pc ? launch_pair_w8<128, 1>(pr, h, st) : launch_pair_w8<128, 2>(pr, h, st);
    default: return cudaErrorInvalidConfiguration;
  }
}

// the fused SwiGLU GEMM covers prefill-sized M (the 2-CTA tiles); below it callers keep the
// GEMM (GEMV / swap-AB tiles) and the separate SwiGLU kernel
constexpr int kSwigluMinM = 256;

// The fused SwiGLU 2-CTA launch (gate/up weight rows interleaved in blocks of 64, N even
// multiple of 64, C [M][N / 2]): width 256 unless 128 fills the clusters better.
cudaError_t run_pair_swiglu(const Problem& pr, int sms, cudaStream_t st) {
  const int P = std::max(1, sms / 2);
  const long long t256 = (long long)((pr.M + 255) / 256) * ((pr.N + 255) / 256);
  const long long t128 = (long long)((pr.M + 255) / 256) * ((pr.N + 127) / 128);
  const double c256 = (double)((t256 + P - 1) / P) * 256.0;
  const double c128 = (double)((t128 + P - 1) / P) * 128.0 / 0.55;
  Hyper h{c128 < c256 ? 128 : 256, 0, 1, 16, 0};
  h.cta_group = 2;
  return h.bn == 256 ? launch_pair<256, true>(pr, h, st) : launch_pair<128, true>(pr, h, st);
}

// Tile widths of the 2-CTA kernel, widest first, and their measured throughput per FLOP
// relative to 256 (narrower tiles read more operand bytes per FLOP from L2; gate_up M = 4096 on
// B200: 224 -> 0.92, 192 -> 0.82, 160 -> 0.67, 128 -> 0.55).
constexpr int kPairBn[] = {256, 224, 192, 160, 128};
constexpr double kPairEff[] = {1.0, 0.92, 0.82, 0.67, 0.55};

// The 2-CTA tile width for an M x N x K problem: the smallest modelled time, pair_plan's cost
// (whole waves, or waves plus a split tail that fits ws_bytes) times bn / 256 / efficiency.
// bn_max caps the choice (the ladder row's bn).
int choose_pair_bn(int M, int N, int K, int sms, int bn_max, size_t ws_bytes, int wkind = 0) {
  if (sms <= 0) return bn_max;  // no device to size waves for
  const int* widths = wkind ? kPairW8Bn : kPairBn;
  const double* eff = wkind ? kPairW8Eff : kPairEff;
  const int nw = wkind ? 2 : 5;
  int best = 0;
  double best_c = 0;
  for (int i = 0; i < nw; ++i) {
    const int bn = widths[i];
    if (bn > bn_max) continue;
    const PairPlan pl = pair_plan(M, N, K, bn, sms, 0, true, ws_bytes);
    const double c = pl.cost * bn / 256.0 / eff[i];
    if (best == 0 || c < best_c) {
      best = bn;
      best_c = c;
    }
  }
  return best;
}

template <int BN>
void pair_facts(int* out6) {
  out6[0] = PairCfg<BN>::THREADS;
  out6[1] = PairCfg<BN>::SMEM;
  out6[2] = PairCfg<BN>::STAGES;
  out6[3] = PairCfg<BN>::TMEM_COLS;
}

int pair_resources(int bn, int* out6) {
  const void* kern = nullptr;
  switch (bn) {
    case 256: kern = reinterpret_cast<const void*>(&k_gemm_sm100_pair<256, false>); pair_facts<256>(out6); break;
    case 224: kern = reinterpret_cast<const void*>(&k_gemm_sm100_pair<224, false>); pair_facts<224>(out6); break;
    case 192: kern = reinterpret_cast<const void*>(&k_gemm_sm100_pair<192, false>); pair_facts<192>(out6); break;
    case 160: kern = reinterpret_cast<const void*>(&k_gemm_sm100_pair<160, false>); pair_facts<160>(out6); break;
    case 128: kern = reinterpret_cast<const void*>(&k_gemm_sm100_pair<128, false>); pair_facts<128>(out6); break;
    default: return cudaErrorInvalidConfiguration;
  }
  cudaFuncAttributes fa{};
  const cudaError_t err = cudaFuncGetAttributes(&fa, kern);
  out6[4] = err == cudaSuccess ? fa.numRegs : -1;
  out6[5] = err == cudaSuccess ? (int)fa.localSizeBytes : -1;
  return err;
}

const InstEntry* find_inst(int wkind, int bn, int swap) {
  for (const auto& e : kInst)
    if (e.wkind == wkind && e.bn == bn && e.swap == swap) return &e;
  return nullptr;
}

// ------------------------------------------------------------------------------------------
// The M-ladder (generated from select.py into dispatch.inc) and the split-K cost model.
// ------------------------------------------------------------------------------------------
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
    if ((N % 16) || !aligned16(scale) || !aligned16(zero)) return false;  // TMA row strides
  }
  return true;
}

// ------------------------------------------------------------------------------------------
// The dispatcher engine: one M-ladder row (generated into dispatch.inc from measured tuner
// rows) plus the problem -> the hyperform to launch.  The k-split comes from a cycle model
// (mirrored by the shipped select.py).
// ------------------------------------------------------------------------------------------
struct LadderRow {
  int m_max;  // inclusive upper bound on M (0x7fffffff = everything else)
  int bn, swap, group_m;
  int cta_group;  // 1, or 2 for the 2-CTA 256 x BN prefill tiles (fp16)
};

// Cycle model of one launch (the busiest SM): waves of units, each k-block costing the larger
// of its UMMAs and its operand feed -- weight bytes stream from HBM at about 32 B/cycle per SM
// (measured TMA streaming rate), activation bytes from L2 at about 100 -- plus the k-split
// fixup: ~1500 cycles through distributed shared memory (splits <= kMaxClusterSplit), the
// fp32 partial round trip through global memory beyond; never below the HBM time
// (compulsory bytes at ~3400 B/cycle for the whole GPU).
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

// The hyperform for `row` of weight kind `wkind` (0 fp16, else a W8 kind); false when the row
// names no instantiation that exists (the caller's fallback).
bool select_hyper(int wkind, const LadderRow& r, int M, int N, int K, size_t ws_bytes, Hyper& h,
                  int sms) {
  h.bn = r.bn;
  h.swap = r.swap;
  h.group_m = r.group_m;
  h.max_ctas = 0;
  h.cta_group = (r.cta_group == 2 && !r.swap) ? 2 : 1;
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
  if (h.cta_group == 2) {  // pair tiles: width and (fp16) split tail by the wave model
    h.bn = choose_pair_bn(M, N, K, sms, h.bn, ws_bytes, wkind);
    h.splits = 2;  // the split tail of pair_plan is allowed
    if (wkind == kWUint8Group && (N % 16)) return false;  // scale/zero rows by TMA
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
  if (h.cta_group == 2) return pr.wkind ? run_pair_w8(pr, h, st) : run_pair(pr, h, st);
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
