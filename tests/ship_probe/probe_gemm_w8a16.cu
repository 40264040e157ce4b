// Host program that builds against a COPY of kernels/shipped/gemm_w8a16/sm_100a alone (its
// launch.cu + this file) and runs the shipped W8A16 path: per-channel int8 and group-wise
// uint8 (group 128) weights, decode, tile and prefill (expanded) sizes; 64 sampled cells
// against an fp64 product on the dequantised weights, relative L2 error over them <= 3e-3.
#include <cmath>
#include <cstdio>
#include <vector>

#include "launch.cuh"

static float h2f(__half h) { return __half2float(h); }

int main() {
  const int shapes[4][3] = {{1, 5120, 5120}, {16, 10240, 5120}, {64, 5120, 8192},
                            {1024, 5120, 4096}};
  int failed = 0;
  for (int kind = TEMPO_W8_INT8_PER_CHANNEL; kind <= TEMPO_W8_UINT8_GROUP; ++kind) {
    for (const auto& s : shapes) {
      const int M = s[0], N = s[1], K = s[2], G = 128, ng = K / G;
      std::vector<__half> a((size_t)M * K), sc(kind == 1 ? N : (size_t)ng * N);
      std::vector<__half> c((size_t)M * N);
      std::vector<uint8_t> w((size_t)N * K), z(kind == 1 ? 0 : (size_t)ng * N);
      for (size_t i = 0; i < a.size(); ++i) a[i] = __float2half(((int)(i % 9) - 4) * 0.25f);
      for (size_t i = 0; i < w.size(); ++i) w[i] = (uint8_t)((i * 2654435761u) >> 24);
      for (size_t i = 0; i < sc.size(); ++i) sc[i] = __float2half(1e-3f + (i % 13) * 1e-3f);
      for (size_t i = 0; i < z.size(); ++i) z[i] = (uint8_t)(100 + i % 57);
      __half *A, *S, *C;
      uint8_t *W, *Z = nullptr;
      void* ws = nullptr;
      cudaMalloc(&A, a.size() * 2);
      cudaMalloc(&S, sc.size() * 2);
      cudaMalloc(&C, c.size() * 2);
      cudaMalloc(&W, w.size());
      cudaMemcpy(A, a.data(), a.size() * 2, cudaMemcpyHostToDevice);
      cudaMemcpy(S, sc.data(), sc.size() * 2, cudaMemcpyHostToDevice);
      cudaMemcpy(W, w.data(), w.size(), cudaMemcpyHostToDevice);
      if (kind == 2) {
        cudaMalloc(&Z, z.size());
        cudaMemcpy(Z, z.data(), z.size(), cudaMemcpyHostToDevice);
      }
      cudaMemset(C, 0x7f, c.size() * 2);
      tempo::gen::W8A16Params p{A, W, S, Z, C, M, N, K, K, K, N, kind, G};
      tempo::gen::Choice ch;
      p.ws_bytes = 1ull << 40;
      const cudaError_t pe = tempo::gen::plan(p, &ch);
      if (ch.ws_bytes) {
        cudaMalloc(&ws, ch.ws_bytes);
        cudaMemset(ws, 0, ch.ws_bytes);
      }
      p.ws = ws;
      p.ws_bytes = ch.ws_bytes;
      const cudaError_t le = tempo::gen::launch(p, 0);
      const cudaError_t se = cudaDeviceSynchronize();
      double worst = 1.0, d2 = 0.0, r2 = 0.0;
      if (le == cudaSuccess && se == cudaSuccess) {
        cudaMemcpy(c.data(), C, c.size() * 2, cudaMemcpyDeviceToHost);
        for (int t = 0; t < 64; ++t) {
          const int m = (t * 37) % M, n = (t * 53) % N;
          double ref = 0.0;
          for (int k = 0; k < K; ++k) {
            const uint8_t q = w[(size_t)n * K + k];
            const double wv = kind == 1 ? (double)(int8_t)q * h2f(sc[n])
                                        : ((double)q - z[(size_t)(k / G) * N + n]) *
                                              h2f(sc[(size_t)(k / G) * N + n]);
            ref += (double)h2f(a[(size_t)m * K + k]) * wv;
          }
          const double d = h2f(c[(size_t)m * N + n]) - ref;
          d2 += d * d;
          r2 += ref * ref;
        }
        worst = r2 > 0 ? sqrt(d2 / r2) : 1.0;
      }
      const bool ok = pe == cudaSuccess && le == cudaSuccess && se == cudaSuccess &&
                      worst <= 3e-3;
      failed += !ok;
      printf("kind=%d M=%-5d N=%-6d K=%-6d bn=%-3d swap=%d expand=%d ws=%zu launch=%s "
             "relL2=%.3e %s\n", kind, M, N, K, ch.bn, ch.swap, ch.expand, ch.ws_bytes,
             cudaGetErrorString(le), worst, ok ? "PASS" : "FAIL");
      cudaFree(A);
      cudaFree(S);
      cudaFree(C);
      cudaFree(W);
      if (Z) cudaFree(Z);
      if (ws) cudaFree(ws);
      if (se != cudaSuccess) return 1;
    }
  }
  printf("SHIPPED PATH: %s\n", failed ? "FAIL" : "PASS");
  return failed ? 1 : 0;
}
