// calib_probes.cu -- measurement probes behind the sm_100a plugin's calibration stage.
//
// The plugin's cost model (estimate_atoms + bound) charges whole-launch loads to channels
// (UMMA, HBM, SMEM_RD, TMA_L2, EPI, DEQ) whose capacities come from measurements.  The copy
// bandwidth and the tensor peak are measured by the build driver; these probes measure the
// rest on the card itself, each as a clock64 period of a loop that does only that channel's
// work, one CTA per SM:
//
//   k_probe_bulk_feed   bulk copies (cp.async.bulk, mbarrier transaction bytes) from global
//                       into a 4-deep shared-memory ring: bytes per cycle per SM from L2 (small
//                       buffer, L2-resident) or from HBM (buffer far larger than L2)
//   k_probe_chase       one thread chasing a pointer ring with L1-bypassing loads: cycles per
//                       dependent load from L2 (ring inside L2) or from HBM (ring far larger)
//   k_probe_dequant     4 warps converting an int8 shared-memory tile to fp16 with the GEMM
//                       kernels' byte-permute method: cycles per element per SM
//   k_probe_store       4 warps storing fp16 rows with 16-byte stores (the epilogue's store
//                       side): bytes per cycle per SM
//
// The reference measures its sm_70 channels with its own stand (tools/probe.cu: a clock64
// period around an unrolled loop, one block per SM) and records them as tempo/calib records
// (tempo/core/calib/schema.py); these probes play that part for sm_100a.  Every wait is bounded
// (%globaltimer, 1 s): on expiry the probe writes ~0ull and returns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace tempo_calib {

constexpr unsigned long long kProbeWaitNs = 1000000000ull;  // 1 s
constexpr int kRing = 4;                                    // bulk-feed ring depth
constexpr int kChunk = 32768;                               // bytes per bulk copy

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool bar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false after kProbeWaitNs.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  if (bar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  while (!bar_try_wait(bar, parity))
    if (gtimer() - t0 > kProbeWaitNs) return false;
  return true;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// One thread per CTA streams `chunks` copies of kChunk bytes, CTA b starting at chunk b and
// striding by the grid, wrapping inside `nchunks`; kRing copies in flight.
__global__ void __launch_bounds__(32) k_probe_bulk_feed(const uint8_t* __restrict__ src,
                                                        long long nchunks, int chunks,
                                                        unsigned long long* out) {
  extern __shared__ __align__(1024) uint8_t ring[];
  __shared__ __align__(8) uint64_t bars[kRing];
  if (threadIdx.x != 0) return;
  for (int s = 0; s < kRing; ++s) bar_init(smem_u32(&bars[s]), 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const unsigned long long t0 = clock64();
  long long c = blockIdx.x;
  bool ok = true;
  for (int i = 0; i < chunks + kRing && ok; ++i) {
    const int s = i % kRing;
    if (i >= kRing) ok = bar_wait(smem_u32(&bars[s]), (uint32_t)(((i / kRing) - 1) & 1));
    if (i < chunks && ok) {
      bar_expect_tx(smem_u32(&bars[s]), kChunk);
      bulk_g2s(smem_u32(ring + s * kChunk), src + (c % nchunks) * kChunk, kChunk,
               smem_u32(&bars[s]));
      c += gridDim.x;
    }
  }
  const unsigned long long t1 = clock64();
  out[blockIdx.x] = ok ? (t1 - t0) : ~0ull;
}

// Pointer chase: next = ring[cur], `steps` times, with ld.global.cg (cached in L2 only).
__global__ void k_probe_chase(const unsigned* __restrict__ ring, int steps,
                              unsigned long long* out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  unsigned cur = 0;
  // warm the first few entries' translations
  for (int i = 0; i < 16; ++i) {
    unsigned v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(ring + cur) : "memory");
    cur = v;
  }
  const unsigned long long t0 = clock64();
  for (int i = 0; i < steps; ++i) {
    unsigned v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(ring + cur) : "memory");
    cur = v;
  }
  const unsigned long long t1 = clock64();
  out[0] = t1 - t0;
  out[1] = cur;  // keeps the chain live
}

// 4 warps convert a 16 KB int8 shared tile to fp16 (32 KB) `iters` times; each lane handles
// 16-byte chunks, as the GEMM kernels' dequant warps do (byte permute into 1024 + b, one half2
// subtraction of the bias 1152 = 1024 + 128 for signed bytes).
__global__ void __launch_bounds__(128) k_probe_dequant(const uint8_t* __restrict__ src, int iters,
                                                        unsigned long long* out) {
  __shared__ __align__(16) uint8_t raw[16384];
  __shared__ __align__(16) __half dst[16384];
  const int t = threadIdx.x;
  for (int i = t * 16; i < 16384; i += 128 * 16)
    *reinterpret_cast<uint4*>(raw + i) = *reinterpret_cast<const uint4*>(src + i);
  __syncthreads();
  const unsigned long long t0 = clock64();
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152.0
  for (int it = 0; it < iters; ++it) {
#pragma unroll 2
    for (int i = t; i < 1024; i += 128) {
      const uint4 x = *reinterpret_cast<const uint4*>(raw + i * 16);
      const uint32_t w[4] = {x.x ^ 0x80808080u, x.y ^ 0x80808080u, x.z ^ 0x80808080u,
                             x.w ^ 0x80808080u};
      uint32_t h[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        h[2 * j] = __byte_perm(w[j], 0x64646464u, 0x5150);
        h[2 * j + 1] = __byte_perm(w[j], 0x64646464u, 0x5352);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        __half2 v = __hsub2(*reinterpret_cast<const __half2*>(&h[j]), bias);
        h[j] = *reinterpret_cast<const uint32_t*>(&v);
      }
      uint4* d = reinterpret_cast<uint4*>(dst + i * 16);
      d[0] = make_uint4(h[0], h[1], h[2], h[3]);
      d[1] = make_uint4(h[4], h[5], h[6], h[7]);
    }
    __syncthreads();
  }
  const unsigned long long t1 = clock64();
  if (t == 0) {
    out[blockIdx.x] = t1 - t0;
    // one converted value, so the loop is not dead code
    out[gridDim.x + blockIdx.x] = __half_as_ushort(dst[blockIdx.x % 16384]);
  }
}

// 4 warps store `bytes_per_cta` of fp16 rows with 16-byte stores into this CTA's slice.
__global__ void __launch_bounds__(128) k_probe_store(uint4* __restrict__ dst,
                                                      long long vec_per_cta,
                                                      unsigned long long* out) {
  uint4* base = dst + (long long)blockIdx.x * vec_per_cta;
  const uint4 v = make_uint4(threadIdx.x, blockIdx.x, 0x3c003c00u, 0x3c003c00u);
  __syncthreads();
  const unsigned long long t0 = clock64();
#pragma unroll 4
  for (long long i = threadIdx.x; i < vec_per_cta; i += 128) base[i] = v;
  __syncthreads();
  const unsigned long long t1 = clock64();
  if (threadIdx.x == 0) out[blockIdx.x] = t1 - t0;
}

}  // namespace tempo_calib

extern "C" {

// Bulk-copy feed: `ctas` CTAs (one per SM) each stream `chunks` copies of 32 KB from `src`
// (`bytes` long, a multiple of 32 KB); cycles_out[ctas] receives each CTA's clock64 period
// (~0 when a wait gave up).  Returns the cudaError_t of the launch and synchronisation.
int tempo_sm100_probe_bulk_feed(const void* src, size_t bytes, int ctas, int chunks,
                                unsigned long long* cycles_out, void* stream) {
  if (!src || bytes < (size_t)tempo_calib::kChunk || ctas <= 0 || chunks <= 0 || !cycles_out)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(src) & 15) return cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int smem = tempo_calib::kRing * tempo_calib::kChunk;
  cudaError_t e = cudaFuncSetAttribute(tempo_calib::k_probe_bulk_feed,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  tempo_calib::k_probe_bulk_feed<<<ctas, 32, smem, st>>>(
      static_cast<const uint8_t*>(src), (long long)(bytes / tempo_calib::kChunk), chunks,
      cycles_out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

// Pointer chase over `ring` (entry i holds the index of the next entry); out2[0] = cycles for
// `steps` dependent loads.
int tempo_sm100_probe_chase(const unsigned* ring, int steps, unsigned long long* out2,
                            void* stream) {
  if (!ring || steps <= 0 || !out2) return cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tempo_calib::k_probe_chase<<<1, 32, 0, st>>>(ring, steps, out2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

// Dequant: `ctas` CTAs of 4 warps convert a 16 KB int8 tile (`src`, 16 KB) `iters` times;
// out[2 * ctas]: per-CTA cycles, then one converted value per CTA.
int tempo_sm100_probe_dequant(const void* src, int ctas, int iters, unsigned long long* out,
                              void* stream) {
  if (!src || ctas <= 0 || iters <= 0 || !out) return cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tempo_calib::k_probe_dequant<<<ctas, 128, 0, st>>>(static_cast<const uint8_t*>(src), iters,
                                                     out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

// Stores: `ctas` CTAs of 4 warps each store `bytes_per_cta` (a multiple of 16) into their own
// slice of `dst` (ctas * bytes_per_cta bytes); out[ctas]: per-CTA cycles.
int tempo_sm100_probe_store(void* dst, size_t bytes_per_cta, int ctas, unsigned long long* out,
                            void* stream) {
  if (!dst || bytes_per_cta < 16 || (bytes_per_cta & 15) || ctas <= 0 || !out)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(dst) & 15) return cudaErrorInvalidValue;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tempo_calib::k_probe_store<<<ctas, 128, 0, st>>>(static_cast<uint4*>(dst),
                                                   (long long)(bytes_per_cta / 16), out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return cudaStreamSynchronize(st);
}

}  // extern "C"
