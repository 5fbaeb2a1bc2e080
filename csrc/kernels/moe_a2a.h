// Expert-parallel dispatch / combine over NVLink peer memory (see moe_a2a.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace a2a {

constexpr int kMaxRanks = 8;

// Symmetric buffers of the exchange, as seen from this rank (index r: the
// buffer on rank r).  `cap` is the most (token, k) pairs a rank sends in one
// layer, so a rank's receive area from one source is cap rows.
struct Args {
  __nv_bfloat16* recv_x[kMaxRanks];          // [world][cap][H] rows received, by source
  int2* recv_meta[kMaxRanks];                // [world][cap] (local expert, source pair index)
  unsigned long long* recv_flag[kMaxRanks];  // [world] (epoch << 32 | pairs sent) per source
  __nv_bfloat16* comb_y[kMaxRanks];          // [cap][H] expert outputs returned, by pair
  unsigned long long* comb_flag[kMaxRanks];  // [world] (epoch << 32 | rows returned) per expert rank
  int* state;                                // local: epoch, then three grid-completion counters
  int* counts;                               // local: [world] pairs sent to each rank, [world] rows received
  int rank, world, experts_local, topk, cap, hidden;
};

// Dispatch: this rank's pairs (ids [T, k] global expert ids) to the ranks that
// hold their experts.  slot: scratch [T * k].
void dispatch(const __nv_bfloat16* h, const int32_t* ids, int T, int32_t* slot, const Args& a, cudaStream_t s);
// Waits for every source, then lays the received rows out in expert order,
// each expert's segment padded to 128 rows: groups [El + 1], perm [rows_max]
// (received row index, -1 for padding), back [rows_max] (source << 32 | pair).
void receive_plan(int32_t* groups, int32_t* perm, long long* back, int rows_max, const Args& a, cudaStream_t s);
// x [rows_max, H] = the received rows in expert order (zeros for padding).
void gather(const int32_t* groups, const int32_t* perm, __nv_bfloat16* x, int rows_max, const Args& a,
            cudaStream_t s);
// Returns each expert output row y [rows_max, H] to its source's combine area.
void combine_send(const __nv_bfloat16* y, const int32_t* groups, const int32_t* perm, const long long* back,
                  const Args& a, cudaStream_t s);
// Waits for every expert rank, then out [T, H] = sum_j w[t, j] * returned row (t, j).
void combine_receive(const float* w, int T, __nv_bfloat16* out, const Args& a, cudaStream_t s);

}  // namespace a2a
}  // namespace lf
