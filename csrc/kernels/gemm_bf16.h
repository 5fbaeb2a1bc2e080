#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "allreduce_ll.h"

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
// Skinny shapes (the plain tiles would leave more than half of the SMs idle)
// run as cluster split-K: one thread-block cluster per output tile, partial
// tiles summed through distributed shared memory, deterministic.  ws is
// accepted for interface stability and unused.
void run(const GemmArgs& a, int epi, int bn, cudaStream_t stream, float* ws = nullptr, int64_t ws_elems = 0);
int plan_splitk(int M, int N, int K, int* kb_per_out);
// The same plan for a device with `sms` multiprocessors.
int plan_splitk_sms(int M, int N, int K, int sms, int* kb_per_out);
// Cluster split-K plan: returns the cluster size (0 = plain tiles) and its BN / k-blocks per CTA /
// 128-row M-blocks per tile.
int plan_cluster(int M, int N, int K, int epi, int* bn_out, int* kb_per_out, int* mb_out = nullptr);
// Enables the 256-row cluster tiles for 129..256-row GEMMs (off by default).
void set_cluster_mb2(int on);
// Enables the single-kernel decode GEMM + low-latency all-reduce in run_allreduce_ll (off by default).
void set_ll_gemm_fused(int on);
// Enables the CTA-pair (tcgen05 cta_group::2) kernel for large GEMMs (on by default).
void set_gemm_pair(int on);
int get_gemm_pair();

// Peer view of one tensor-parallel group for the fused GEMM + all-reduce.
// Two symmetric bf16 regions of [rows, N] (every rank holds both, same size):
// `local`/`mc`/`peer[r]` address this rank's partial-sum region (own address,
// NVLink multicast address or null, address on rank r); `out_mc`/`out_peer[r]`
// address the result region, which is the operation's output on every rank.
// A piece (an output tile, or a group of rows) has one owner rank: every rank
// publishes its partial of the piece and signals the owner; the owner reads
// the sum of all partials through the switch (multimem.ld_reduce) and writes
// it into every rank's result region (multimem.st), then signals "done" to
// every rank.  Each rank's NVLink traffic is then about twice the output size,
// independent of the group size (a bandwidth-optimal all-reduce).
// `cnt_*` address int32 counters: [0, cnt_capacity) arrivals, then
// [cnt_capacity, 2 cnt_capacity) completions; every wait re-arms its counter.
constexpr int kMaxRanks = 8;

// QKV projection epilogue (kQkvRope): the output columns are Hq query heads,
// then Hkv key heads, then Hkv value heads, 128 wide each.  Query heads are
// rotated (split-half RoPE, angles from cos_sin [max_pos][64] (cos, sin)) and
// written to D; key heads are rotated and value heads copied into the paged
// cache ([page][kv_head][page_size][128] per K / V) at slots[row] (negative:
// no write).  D's key / value columns are not written.
struct RopeArgs {
  const int32_t* positions;
  const int32_t* slots;
  const float2* cos_sin;
  __nv_bfloat16* kcache;
  __nv_bfloat16* vcache;
  int Hq, Hkv, page, max_pos;
  int64_t num_slots;
};

struct ArArgs {
  __nv_bfloat16* local;
  __nv_bfloat16* mc;
  const __nv_bfloat16* peer[kMaxRanks];
  __nv_bfloat16* out_mc;
  __nv_bfloat16* out_peer[kMaxRanks];
  int* cnt_local;
  int* cnt_mc;
  int* cnt_peer[kMaxRanks];
  int rank;
  int world;
  int cnt_capacity;
  // Optional timeline (null in production): per tile, %globaltimer at
  // [4 t] partial published, [4 t + 1] owner saw every partial, [4 t + 2]
  // owner's sum written everywhere; [4 t + 3] = 1 + the owner CTA's index.
  unsigned long long* trace;
  // Reduce-scatter mode (rs_rows > 0): rank r owns output rows
  // [r rs_rows, (r + 1) rs_rows) (tiles are dealt by rows, rs_rows a multiple
  // of 128), and the owner writes its sums only to rs_out ([rs_rows, N], row
  // stride N) instead of every rank's result region.
  int rs_rows;
  __nv_bfloat16* rs_out;
};

// Sum of `splits` fp32 [M, N] slabs in ws, then the sum over the group, into
// the result region (the split-K finalize kernel with its fused all-reduce).
void partials_allreduce(const float* ws, int M, int N, int splits, const ArArgs& ar, cudaStream_t stream);
// align: the segments' row multiple (128, or 256: CTA-pair tiles, one expert per 256-row tile).
void run_grouped(const GemmArgs& a, const int* groups, int num_groups, int epi, cudaStream_t stream,
                 int align = 128);
// Result region = sum over the tensor-parallel group of this rank's A . B^T,
// computed and all-reduced over NVLink by one kernel (split-K shapes: the GEMM
// and the finalize kernel that carries the all-reduce).  a.D is unused.
void run_allreduce(const GemmArgs& a, const ArArgs& ar, cudaStream_t stream, float* ws, int64_t ws_elems);
// The row-parallel GEMM fused with a reduce-scatter by rows (ar.rs_rows,
// ar.rs_out set; M == rs_rows * world): the owner-computes tile path with the
// result kept by the owner.
void run_reduce_scatter(const GemmArgs& a, const ArArgs& ar, cudaStream_t stream);
int choose_bn(int M, int N, int epi);
int choose_bn_sms(int M, int N, int epi, int sms);
// Decode shapes: GEMM into fp32 slabs of ws (split-K when it fills the SMs),
// then the low-latency all-reduce (allreduce_ll.h) into a.D.
void run_allreduce_ll(const GemmArgs& a, const ar::LLArgs& ll, cudaStream_t stream, float* ws, int64_t ws_elems);
// QKV projection with RoPE and the paged K / V write in the epilogue (see
// RopeArgs; D is [M, (Hq + 2 Hkv) * 128]).  Returns false, having launched
// nothing, when the shape has no tile plan with whole heads per tile.
bool run_qkv_rope(const GemmArgs& a, const RopeArgs& rope, cudaStream_t stream);

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                         uint64_t cols, uint64_t ld_elems, uint32_t box_rows, uint32_t box_cols,
                         CUtensorMapSwizzle swizzle);

}  // namespace gemm
}  // namespace lf
