#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace gemm {

struct GemmArgs {
  const void* A;   // [M, K] bf16, row stride lda (elements)
  const void* B;   // [N, K] bf16, row stride ldb (elements)
  void* D;         // [M, N] (bf16 or fp32), row stride ldd; [M, N/2] for SwiGLU
  int M, N, K;
  int64_t lda, ldb, ldd;
};

// epi: 0 = bf16 store, 1 = fp32 store, 2 = SwiGLU (gate/up rows interleaved in
// groups of 64: 32 gate rows then the matching 32 up rows).  bn = 0 picks a tile width from the shape.
// ws: optional fp32 scratch of ws_elems floats; when given and the GEMM is
// too skinny to fill the SMs, the K dimension is split, each split writes its
// own [M, N] slab of ws and a finalize kernel sums the slabs in split order
// (deterministic; needs splits * M * N <= ws_elems, else no split).
void run(const GemmArgs& a, int epi, int bn, cudaStream_t stream, float* ws = nullptr, int64_t ws_elems = 0);
int plan_splitk(int M, int N, int K, int* kb_per_out);

// Peer view of one tensor-parallel group for the fused GEMM + all-reduce
// epilogue.  `local` is this rank's slot of a symmetric (every rank holds one,
// same size) bf16 buffer [rows, N]; `mc` is the NVLink-multicast address of
// the same slot (null when the fabric has no multicast); `peer[r]` are the
// slot's addresses on every rank.  `cnt_*` are per-tile int32 arrival counters
// laid out the same way.
constexpr int kMaxRanks = 8;
struct ArArgs {
  __nv_bfloat16* local;
  __nv_bfloat16* mc;
  const __nv_bfloat16* peer[kMaxRanks];
  int* cnt_local;
  int* cnt_mc;
  int* cnt_peer[kMaxRanks];
  int world;
  int cnt_capacity;
};

// D = sum over the tensor-parallel group of this rank's A . B^T, computed and
// all-reduced by one kernel over NVLink (see ArArgs).
// Sum of `splits` fp32 [M, N] slabs in ws, then the sum over the group, into
// bf16 D (the split-K finalize kernel with its fused all-reduce).
void partials_allreduce(const float* ws, void* D, int M, int N, int64_t ldd, int splits, const ArArgs& ar,
                        cudaStream_t stream);
void run_grouped(const GemmArgs& a, const int* groups, int num_groups, int epi, cudaStream_t stream);
void run_allreduce(const GemmArgs& a, const ArArgs& ar, cudaStream_t stream, float* ws, int64_t ws_elems);
int choose_bn(int M, int N, int epi);

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                         uint64_t cols, uint64_t ld_elems, uint32_t box_rows, uint32_t box_cols,
                         CUtensorMapSwizzle swizzle);

}  // namespace gemm
}  // namespace lf
