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
// ws: an all-zero fp32 workspace of ws_elems (>= M * N for split-K; null or
// too small: no split); it is all-zero again when the GEMM has run.
void run(const Fp8Args& a, int epi, cudaStream_t s, float* ws = nullptr, int64_t ws_elems = 0);
// K splits for `tiles` output tiles over num_kb 128-wide K blocks on `sms`
// SMs (1: no split); *kb_per receives the K blocks per split.
int plan_splits(int tiles, int num_kb, int sms, int* kb_per);
// Per-token, per-128-channel e4m3 quantisation of a bf16 activation.
void act_quant(const void* x, int64_t ldx, int M, int K, void* q, float* s, int64_t lds, cudaStream_t st);

}  // namespace fp8
}  // namespace lf
