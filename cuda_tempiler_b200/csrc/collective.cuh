// One-shot all-reduce (sum) of an fp16 vector over the ranks of a tensor-parallel group on one
// node, through peer memory (CUDA IPC mappings over NVLink / NVSwitch): the decode-sized
// exchange of the row-parallel down projection, where NCCL's ring/tree latency dominates.
//
// Every rank owns a receive buffer [2][tp][cap] fp16 (two halves alternate by call parity) and
// a flag array [tp][kArMaxCtas] uint32, both mapped into every peer.  CTA b of rank r:
//   1. stores its slice of r's vector into slot r of every rank's receive buffer (peer stores);
//   2. after a CTA barrier, writes `epoch` into flag [r][b] of every rank with a system-scope
//      release store;
//   3. waits (bounded) until flag [s][b] of its own array reads `epoch` for every rank s;
//   4. sums slots 0 .. tp-1 of its slice in rank order (the same order on every rank, so all
//      ranks hold bit-identical results) and writes the output.
// Two halves suffice: a rank starts call k + 2 only after every rank has stored for call k + 1,
// which each does only after finishing call k.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace tempo_sm100 {

constexpr int kArMaxTp = 8;
constexpr int kArMaxCtas = 32;

struct PeerSet {
  __half* recv[kArMaxTp];     // rank p's receive buffer, as mapped in this process
  uint32_t* flags[kArMaxTp];  // rank p's flag array, as mapped in this process
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// src and dst may be the same buffer (an in-place all-reduce): neither is __restrict__.  Each
// thread reads src[v] and later writes dst[v] only for its own v, after a __syncthreads, so
// aliasing is safe.  wait_ns bounds the flag wait (2 s in the public entry point).
__global__ void __launch_bounds__(256)
    k_allreduce_oneshot(const __half* src, __half* dst, long long n, long long cap,
                        const __grid_constant__ PeerSet peers, int tp, int rank, uint32_t epoch,
                        unsigned long long wait_ns, uint32_t* dev_epoch) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // src comes from the preceding GEMM
  // Device-side epoch (dev_epoch != nullptr): [0] the last completed epoch, [1] CTAs done with
  // the current call.  Every CTA reads [0] before it arrives on [1], and only the last CTA to
  // arrive advances [0], so all CTAs of a call use the same epoch, and a call captured in a
  // CUDA graph gets a new epoch on every replay.
  if (dev_epoch) epoch = *reinterpret_cast<volatile uint32_t*>(dev_epoch) + 1u;
  const long long nv = n / 8;  // 16-byte vectors
  const long long per = (nv + gridDim.x - 1) / gridDim.x;
  const long long v0 = (long long)blockIdx.x * per;
  const long long v1 = v0 + per < nv ? v0 + per : nv;
  const long long half_off = (long long)(epoch & 1u) * tp * cap;
  const uint4* s = reinterpret_cast<const uint4*>(src);
  // 1. this rank's slice into slot `rank` of every rank
  for (int p = 0; p < tp; ++p) {
    uint4* d = reinterpret_cast<uint4*>(peers.recv[p] + half_off + (long long)rank * cap);
    for (long long v = v0 + threadIdx.x; v < v1; v += blockDim.x) d[v] = s[v];
  }
  // the CTA barrier orders every thread's slot stores before the flag stores below, and a
  // release store is cumulative: a peer that acquires the flag sees the whole slice
  __syncthreads();
  // 2. announce it
  if (threadIdx.x < tp)
    st_release_sys(peers.flags[threadIdx.x] + rank * kArMaxCtas + blockIdx.x, epoch);
  // 3. wait for every rank's slice (bounded; a missing rank leaves an error status)
  if (threadIdx.x < tp) {
    const uint32_t* f = peers.flags[rank] + threadIdx.x * kArMaxCtas + blockIdx.x;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) != epoch) {
      if (globaltimer() - t0 > wait_ns) {
        if (atomicCAS(&g_status[0], 0, 1) == 0) {
          g_status[1] = 20;  // all-reduce wait
          g_status[2] = blockIdx.x;
          g_status[3] = threadIdx.x;
        }
        break;
      }
    }
  }
  __syncthreads();
  // 4. sum the slots in rank order
  const __half* base = peers.recv[rank] + half_off;
  uint4* o = reinterpret_cast<uint4*>(dst);
  for (long long v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < tp; ++q) {
      const uint4 x = reinterpret_cast<const uint4*>(base + (long long)q * cap)[v];
      const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    uint4 r;
    __half2* rh = reinterpret_cast<__half2*>(&r);
#pragma unroll
    for (int j = 0; j < 4; ++j) rh[j] = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);
    o[v] = r;
  }
  if (dev_epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(dev_epoch + 1, 1u) == gridDim.x - 1) {
        dev_epoch[1] = 0;
        __threadfence();
        atomicExch(dev_epoch, epoch);
      }
    }
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace tempo_sm100
