/* tempo_sm100.h -- C-ABI of the sm_100a (B200) GEMM backend of the tempolator.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed as void*,
 * and returns an int that is a cudaError_t value.  Semantics follow the reference's shipped
 * POD ABI (kernels/shipped/gemm_fp16/sm_70/launch.cuh:20-75, launch.cu:20-22,
 * dispatch.inc:15-26):
 *
 *   0  (cudaSuccess)                    the kernel was launched on `stream`
 *   9  (cudaErrorInvalidConfiguration)  "not covered": the caller must take its own fallback
 *                                       path (F.linear / cuBLAS), exactly like the reference
 *                                       dispatcher's last line (dispatch.inc:26)
 *   other                               a real CUDA error
 *
 * Layouts (the reference's k/k/n layout, kernels/naive/gemm_fp16.cu:16-38):
 *   A [M][K] fp16, row stride lda;   B [N][K] fp16, row stride ldb;   C [M][N] fp16, ldc.
 *   C = A * B^T with fp32 accumulation.  Strides are in elements and must be multiples of
 *   8 (16 bytes); base pointers 16-byte aligned; K and N multiples of 8.
 *
 * Workspace: split-K launches need `ws` (device memory, zero-filled once by the caller before
 * its first use).  Its first 64 KiB hold arrival counters, which every launch leaves at zero
 * and nothing else ever writes; the rest holds fp32 partials (and, for the W8A16 prefill, the
 * fp16 copy of the weights right after the counters), which need no clearing.  Query the size with
 * tempo_sm100_workspace_bytes.  ws == NULL or too small is legal: the dispatcher then picks
 * a configuration without split-K.  A non-NULL ws must be 16-byte aligned (else 1,
 * cudaErrorInvalidValue, and nothing is launched).  One workspace must not be shared by
 * launches that can run concurrently (different streams).
 *
 * Threading: all entry points are re-entrant; per-device one-time set-up is internal.
 */
#ifndef TEMPO_SM100_H
#define TEMPO_SM100_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight quantisation kinds for the W8A16 op. */
#define TEMPO_W8_INT8_PER_CHANNEL 1  /* int8 W [N][K], fp16 scale [N]; W = q * s[n]           */
#define TEMPO_W8_UINT8_GROUP 2       /* uint8 W [N][K], fp16 scale/uint8 zero [K/g][N] (GPTQ's
                                        scales and byte view of qzeros); W = (q - z) * s      */

/* Replaces tempo::gen::applicable(const GemmParams&) (launch.cuh:59-67).  1 = covered.
 * The C-ABI is a thin layer over the shipped POD ABI (kernels/shipped/<op>/sm_100a/launch.cuh:
 * tempo::gen::GemmParams / W8A16Params, applicable(), launch(), plan()), for callers that bind
 * C symbols (ctypes, cgo, JNI) rather than compile the ship directory into their own tree. */
int tempo_sm100_gemm_fp16_applicable(const void* A, const void* B, const void* C, int M, int N,
                                     int K, int lda, int ldb, int ldc);

/* Replaces tempo::gen::launch(const GemmParams&, cudaStream_t) (launch.cuh:75, launch.cu:20-22):
 * C[M][N] = A[M][K] * B[N][K]^T, fp16 in/out, fp32 accumulate, tcgen05 tensor cores. */
int tempo_sm100_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, int lda,
                          int ldb, int ldc, void* ws, size_t ws_bytes, void* stream);

/* The W8A16 op (north-star skeleton gemm_w8a16; the reference's unshipped sm70 skeleton is
 * tempo/plugins/sm70/skeletons/gemm_w8a16/kernel.cuh:226-296, its GPTQ reconstruction formula
 * bench/gemm_baseline.py:214-231).  W is [N][K] 8-bit, row stride ldw (bytes, multiple of 16).
 * quant_kind TEMPO_W8_INT8_PER_CHANNEL: scale [N], zero ignored, group_size ignored.
 * quant_kind TEMPO_W8_UINT8_GROUP: scale fp16 [K/group_size][N], zero uint8 [K/group_size][N]
 * (GPTQ's scales array and the byte view of its qzeros, zero-copy), group_size a multiple of 64
 * dividing K, N a multiple of 16, scale and zero 16-byte aligned. */
int tempo_sm100_gemm_w8a16_applicable(const void* A, const void* W, const void* scale,
                                      const void* zero, const void* C, int M, int N, int K,
                                      int lda, int ldw, int ldc, int quant_kind, int group_size);
/* From M = 1024 on, given a workspace of at least 65536 + N * K * 2 bytes
 * (tempo_sm100_workspace_bytes asks for it), the weights are first expanded to fp16 in the
 * workspace by an HBM-bound pass and the fp16 2-CTA kernel runs on the copy; below that, or
 * with less workspace, the 8-bit weights are dequantised inside the tensor-core kernel (or the streaming GEMV for M <= 16). */
int tempo_sm100_gemm_w8a16(const void* A, const void* W, const void* scale, const void* zero,
                           void* C, int M, int N, int K, int lda, int ldw, int ldc, int quant_kind,
                           int group_size, void* ws, size_t ws_bytes, void* stream);

/* Workspace bytes the dispatcher would like for this problem (0 = no split-K wanted).
 * weight_kind: 0 = fp16, else a TEMPO_W8_* kind. */
size_t tempo_sm100_workspace_bytes(int M, int N, int K, int weight_kind);

/* One explicit hyperform (the plugin's search axes; used by the build/measure stages and the
 * tuner).  bn: MMA N tile (16..256), swap: 1 = weights on the 128-row MMA side (8-bit weights
 * dequantised into TMEM), 2 = the same with 8-bit weights dequantised into shared memory
 * (weight_kind 1 or 2, bn 32 / 64 / 128), splits: k-split
 * count (1 = none), group_m: raster group height in 128-row tiles, max_ctas: persistent grid
 * cap (0 = one CTA per SM).  Returns 9 if the hyperform is not instantiated or does not fit. */
int tempo_sm100_gemm_hyperform(int weight_kind, const void* A, const void* W, const void* scale,
                               const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                               int ldc, int group_size, int bn, int swap, int splits, int group_m,
                               int max_ctas, void* ws, size_t ws_bytes, void* stream);

/* As tempo_sm100_gemm_hyperform with the cluster axis: cta_group 2 runs prefill tiles of
 * 256 x bn on 2-CTA clusters with tcgen05.mma.cta_group::2 (swap 0): fp16 weights with bn
 * 128..256 step 32, 8-bit weights (dequantised in shared memory by each CTA) with bn 128 or
 * 256.  There splits 1 = one cluster per tile; splits > 1 lets a ragged last wave run as
 * a split tail (its tiles cut into k-slices, reduced in k order by the last slice; needs up to
 * 65536 + 3 * P * 2 * 128 * bn * 4 bytes of workspace for P = SMs / 2 clusters, else the
 * launch stays data-parallel).  cta_group 1 is tempo_sm100_gemm_hyperform. */
int tempo_sm100_gemm_hyperform_cg(int weight_kind, const void* A, const void* W, const void* scale,
                                  const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                                  int ldc, int group_size, int bn, int swap, int splits,
                                  int group_m, int max_ctas, int cta_group, void* ws,
                                  size_t ws_bytes, void* stream);

/* Resource facts of the 2-CTA instantiation k_gemm_sm100_pair<bn>, laid out as
 * tempo_sm100_hyperform_resources' out6 (per CTA). */
int tempo_sm100_pair_resources(int bn, int* out6);

/* The dispatcher's choice for a problem: out[0..4] = bn, swap, splits, group_m, stages.
 * Returns 9 if the problem is not covered. */
int tempo_sm100_select(int weight_kind, int M, int N, int K, size_t ws_bytes, int* out5);

/* Resource facts of one instantiation: out[0..5] = threads, dynamic smem bytes, stages,
 * TMEM columns, registers per thread, local (stack/spill) bytes per thread.  Non-zero return
 * if the instantiation does not exist. */
int tempo_sm100_hyperform_resources(int weight_kind, int bn, int swap, int* out6);

/* The naive INPUT bar (one thread per output, fp32 accumulate) -- the reference's
 * kernels/naive/gemm_fp16.cu:60-76 operation, and its W8A16 analogue. */
int tempo_sm100_naive_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K,
                                int lda, int ldb, int ldc, void* stream);
int tempo_sm100_naive_gemm_w8a16(const void* A, const void* W, const void* scale,
                                 const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                                 int ldc, int quant_kind, int group_size, void* stream);

/* out[m][i] = silu(gate) * up for a gate_up GEMM output row m (the SwiGLU step of the
 * tensor-parallel MLP; the reference names this elementwise cost but has no kernel for it).
 * block 0: the row holds the gate half [0, I) and the up half [I, 2I); block b > 0: gate and
 * up alternate in blocks of b columns (the interleaved layout of the fused entry points below).
 * fp16, I % 8 == 0, b % 8 == 0 and I % b == 0. */
int tempo_sm100_silu_mul(const void* gu, void* out, int M, int I, int ld_gu, int ld_out,
                         int block, void* stream);

/* gate_up GEMM with the SwiGLU step fused into its epilogue (reference: the fusion its notes
 * name as next, tempo/plugins/sm70/__init__.py:66).  W [N][K] holds the gate and up weight rows
 * interleaved in blocks of 64 (rows 128 t + j: gate row 64 t + j; rows 128 t + 64 + j: up row
 * 64 t + j), N = 2 I a multiple of 128; C [M][I] = silu(A Wg^T) * (A Wu^T), ldc >= I.  Covers
 * M > 256 (2-CTA tiles); 9 below, where the GEMM plus tempo_sm100_silu_mul (block 64) is the
 * caller's path.  The W8A16 form (same quantisation arguments as tempo_sm100_gemm_w8a16, scales
 * and zero points permuted like the rows) covers M >= 512 with ws >= 65536 + N * K * 2 bytes. */
int tempo_sm100_gemm_fp16_swiglu(const void* A, const void* W, void* C, int M, int N, int K,
                                 int lda, int ldw, int ldc, void* stream);
int tempo_sm100_gemm_w8a16_swiglu(const void* A, const void* W, const void* scale,
                                  const void* zero, void* C, int M, int N, int K, int lda, int ldw,
                                  int ldc, int quant_kind, int group_size, void* ws,
                                  size_t ws_bytes, void* stream);

/* Peer memory for the tensor-parallel exchange (one process per GPU of one node): a zeroed
 * device allocation of its own (an IPC handle maps a whole allocation, so the buffers must not
 * be sub-allocations of a caching allocator) and its release, the 64-byte CUDA IPC handle of
 * such an allocation, its mapping in another process, and the unmapping. */
#define TEMPO_SM100_IPC_HANDLE_BYTES 64
int tempo_sm100_ipc_alloc(size_t bytes, void** out_ptr);
int tempo_sm100_ipc_free(void* ptr);
int tempo_sm100_ipc_handle(const void* dptr, void* out_handle);
int tempo_sm100_ipc_open(const void* handle, void** out_ptr);
int tempo_sm100_ipc_close(void* ptr);

/* One-shot all-reduce (sum) of n fp16 values over tp <= 8 ranks through peer memory, for the
 * decode-sized partial of the row-parallel down projection (no counterpart in the reference,
 * which is single-GPU; NCCL's all-reduce is the general path).  recv[p] / flags[p]: rank p's
 * receive buffer (2 * tp * cap fp16, 16-byte aligned) and flag array (tp * 32 uint32, zeroed
 * once), as mapped in this process (this rank's own at p == rank).  epoch: 1, 2, 3, ... per
 * call, the same on every rank.  ctas <= 32 CTAs split the vector.  Every rank must make the
 * same call; a rank that does not arrive within 2 s leaves status 1 (role 20) in
 * tempo_sm100_device_status and the output undefined.  n % 8 == 0, n <= cap. */
int tempo_sm100_allreduce_oneshot(const void* src, void* dst, long long n, long long cap,
                                  void* const* recv, void* const* flags, int tp, int rank,
                                  unsigned epoch, int ctas, void* stream);
/* The same with the flag wait bounded by wait_ns (1 .. 2e9 ns) instead of 2 s: a rank that
 * has not arrived by then leaves status 1, role 20 and the output undefined.  For callers
 * that want a faster failure report than 2 s (and for the test that makes the wait run out). */
int tempo_sm100_allreduce_oneshot_timed(const void* src, void* dst, long long n, long long cap,
                                        void* const* recv, void* const* flags, int tp, int rank,
                                        unsigned epoch, int ctas, unsigned long long wait_ns,
                                        void* stream);

/* The same with the epoch kept on the device: epoch_ctr is this rank's own buffer of two
 * uint32 (8-byte aligned, zeroed once), which the kernel reads and advances itself, so the
 * call can be captured in a CUDA graph and replayed (every rank must replay in step).  Do not
 * mix it with explicit-epoch calls on the same buffers. */
int tempo_sm100_allreduce_oneshot_dev(const void* src, void* dst, long long n, long long cap,
                                      void* const* recv, void* const* flags, int tp, int rank,
                                      void* epoch_ctr, int ctas, void* stream);

/* Device status written by bounded waits inside the kernels: out[0] = 0 ok / 1 timeout,
 * out[1] = role that gave up, out[2] = block.  reset != 0 clears it.  Synchronises the
 * current device. */
int tempo_sm100_device_status(int* out4, int reset);

/* Allocation-free variant of tempo_sm100_gemm_fp16 (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory for this library: serving frameworks that
 * reserve nearly all HBM for their own caching allocator (a foreign cudaMalloc fails or
 * fragments their pool), latency-critical paths where cudaMalloc/cudaFree would implicitly
 * synchronise the device, and FFI callers with no device allocator to provide a workspace.
 * The caller still passes A, B and C; the split-K scratch is a fixed device array of
 * TEMPO_SM100_NOALLOC_SCRATCH_BYTES inside the library, held by every GPU that loads it until
 * the process exits.  Never calls cudaMalloc, cudaFree or any allocating routine.
 *
 * - The first call on a device resolves the array's device address (cudaGetSymbolAddress, with
 *   that device current); make that first call before any stream capture on the device.
 * - Picks the same configuration as tempo_sm100_gemm_fp16 with a full-size workspace; if that
 *   configuration needs more scratch than TEMPO_SM100_NOALLOC_SCRATCH_BYTES (see
 *   tempo_sm100_workspace_bytes) the call is rejected with 1 (cudaErrorInvalidValue) and
 *   launches nothing.
 * - All calls on a device share the one array and it keeps the last call's contents (the
 *   counters are cleared on the stream before each launch): calls that may overlap on the GPU
 *   (different streams, or concurrent host threads) race and must be serialised by the caller. */
#define TEMPO_SM100_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)
int tempo_sm100_gemm_fp16_noalloc(const void* A, const void* B, void* C, int M, int N, int K,
                                  int lda, int ldb, int ldc, void* stream);

/* ---- calibration probes (the plugin's `calibrate` stage) ----------------------------------
 * Replace the reference's measurement stand for its sm_70 channel rates (tools/probe.cu: a
 * clock64 period around a loop doing one channel's work, one block per SM, recorded as
 * tempo/calib records -- tempo/core/calib/schema.py:19-33).  Each runs one launch, synchronises
 * `stream` and returns the cudaError_t; per-CTA clock64 periods go to the caller's DEVICE
 * buffer (~0 when a bounded wait gave up).  They allocate nothing.
 *
 * Bulk-copy feed into shared memory: `ctas` CTAs each stream `chunks` 32 KB copies from `src`
 * (`bytes`, >= 32 KB, 16-byte aligned), 4 in flight.  cycles_out[ctas]. */
int tempo_sm100_probe_bulk_feed(const void* src, size_t bytes, int ctas, int chunks,
                                unsigned long long* cycles_out, void* stream);
/* One thread chasing `ring` (ring[i] = next index) for `steps` L1-bypassing loads;
 * out2[0] = cycles. */
int tempo_sm100_probe_chase(const unsigned* ring, int steps, unsigned long long* out2,
                            void* stream);
/* `ctas` CTAs of 4 warps converting a 16 KB int8 tile (`src`) to fp16 `iters` times, the GEMM
 * kernels' conversion; out[2 * ctas]: cycles per CTA, then one converted value per CTA. */
int tempo_sm100_probe_dequant(const void* src, int ctas, int iters, unsigned long long* out,
                              void* stream);
/* `ctas` CTAs of 4 warps storing `bytes_per_cta` (multiple of 16) with 16-byte stores into
 * their own slices of `dst`; out[ctas]: cycles per CTA. */
int tempo_sm100_probe_store(void* dst, size_t bytes_per_cta, int ctas, unsigned long long* out,
                            void* stream);

/* Library identification string. */
const char* tempo_sm100_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TEMPO_SM100_H */
