// Host program that builds against a COPY of kernels/shipped/gemm_fp16/sm_100a alone (its
// launch.cu + this file, nothing else of the repository) and runs the shipped path on the
// reference ship probe's patterned inputs: A = ((i % 7) - 3) / 8, B = ((i % 5) - 2) / 8, six
// shapes, 64 sampled cells against an fp64 dot product, max |got - ref| / (|ref| + 1e-3) <= 3e-3
// (kernels/shipped/gemm_fp16/sm_70/ship_probe.cu:35-99).  C is poisoned with 0x7f7f first.
#include <cmath>
#include <cstdio>
#include <vector>

#include "launch.cuh"

int main() {
  const int shapes[6][3] = {{1, 4096, 3840},  {8, 4096, 3840},   {32, 15360, 3840},
                            {128, 4096, 3840}, {512, 15360, 3840}, {2048, 3840, 15360}};
  int failed = 0;
  for (const auto& s : shapes) {
    const int M = s[0], N = s[1], K = s[2];
    std::vector<__half> a((size_t)M * K), b((size_t)N * K), c((size_t)M * N);
    for (size_t i = 0; i < a.size(); ++i) a[i] = __float2half(((int)(i % 7) - 3) * 0.125f);
    for (size_t i = 0; i < b.size(); ++i) b[i] = __float2half(((int)(i % 5) - 2) * 0.125f);
    __half *A, *B, *C;
    void* ws = nullptr;
    cudaMalloc(&A, a.size() * 2);
    cudaMalloc(&B, b.size() * 2);
    cudaMalloc(&C, c.size() * 2);
    cudaMemcpy(A, a.data(), a.size() * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(B, b.data(), b.size() * 2, cudaMemcpyHostToDevice);
    cudaMemset(C, 0x7f, c.size() * 2);
    tempo::gen::GemmParams p{A, B, C, M, N, K, K, K, N};
    tempo::gen::Choice ch;
    p.ws_bytes = 1ull << 40;  // plan with any workspace, then give it what it asks for
    const cudaError_t pe = tempo::gen::plan(p, &ch);
    p.ws_bytes = ch.ws_bytes;
    if (ch.ws_bytes) {
      cudaMalloc(&ws, ch.ws_bytes);
      cudaMemset(ws, 0, ch.ws_bytes);
    }
    p.ws = ws;
    const bool app = tempo::gen::applicable(p);
    const cudaError_t le = tempo::gen::launch(p, 0);
    const cudaError_t se = cudaDeviceSynchronize();
    double worst = 0.0;
    if (le == cudaSuccess && se == cudaSuccess) {
      cudaMemcpy(c.data(), C, c.size() * 2, cudaMemcpyDeviceToHost);
      for (int t = 0; t < 64; ++t) {
        const int m = (t * 37) % M, n = (t * 53) % N;
        double ref = 0.0;
        for (int k = 0; k < K; ++k)
          ref += (double)__half2float(a[(size_t)m * K + k]) * __half2float(b[(size_t)n * K + k]);
        const double got = __half2float(c[(size_t)m * N + n]);
        worst = fmax(worst, fabs(got - ref) / (fabs(ref) + 1e-3));
      }
    }
    const bool ok = pe == cudaSuccess && app && le == cudaSuccess && se == cudaSuccess &&
                    worst <= 3e-3;
    failed += !ok;
    printf("M=%-5d N=%-6d K=%-6d bn=%-3d swap=%d cta_group=%d ws=%zu launch=%s sync=%s "
           "maxrel=%.3e %s\n", M, N, K, ch.bn, ch.swap, ch.cta_group, ch.ws_bytes,
           cudaGetErrorString(le), cudaGetErrorString(se), worst, ok ? "PASS" : "FAIL");
    cudaFree(A);
    cudaFree(B);
    cudaFree(C);
    if (ws) cudaFree(ws);
    if (se != cudaSuccess) break;  // the context is gone; later shapes would not mean anything
  }
  // a problem the dispatcher does not cover answers cudaErrorInvalidConfiguration
  tempo::gen::GemmParams bad{nullptr, nullptr, nullptr, 4, 4095, 3840, 3840, 3840, 4095};
  if (tempo::gen::launch(bad, 0) != cudaErrorInvalidConfiguration) ++failed;
  printf("SHIPPED PATH: %s\n", failed ? "FAIL" : "PASS");
  return failed ? 1 : 0;
}
