#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace fp8 {

struct Fp8Args {
  const void* A;      // e4m3 [M, K], row stride lda (bytes == elements)
  const void* B;      // e4m3 [N, K], row stride ldb
  const float* sa;    // [M, K / 128] activation scales, row stride lds_a
  int64_t lds_a;
  const float* sb;    // [N / 128, K / 128] weight block scales
  void* D;            // [M, N] bf16 / fp32, or [M, N / 2] bf16 for SwiGLU
  int M, N, K;
  int64_t lda, ldb, ldd;
};

// epi: 0 bf16, 1 fp32, 2 SwiGLU (gate/up rows interleaved in groups of 32).
void run(const Fp8Args& a, int epi, cudaStream_t s);
// Per-token, per-128-channel e4m3 quantisation of a bf16 activation.
void act_quant(const void* x, int64_t ldx, int M, int K, void* q, float* s, int64_t lds, cudaStream_t st);

}  // namespace fp8
}  // namespace lf
