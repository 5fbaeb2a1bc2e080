// Low-latency all-reduce of fp32 partial sums over NVLink (decode shapes).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace ar {

constexpr int kMaxRanks = 8;

// Inboxes of the low-latency protocol, in symmetric memory (same offsets on
// every rank).  Every 8-byte word carries two bf16 values and the operation's
// epoch, written by ONE store, so a reader that sees the epoch sees the data:
// no fence, no separate flag, no round trip.
//   rs[r]  inbox of rank r for the reduce-scatter step: [world][chunk] words
//   ag[r]  inbox of rank r for the all-gather step: [pairs] words
//   ag_mc  NVLink multicast address of the all-gather inboxes (null when the
//          fabric has none): one store reaches every rank
//   state  this rank's (epoch, finished CTAs), in local memory
struct LLArgs {
  uint2* rs[kMaxRanks];
  uint2* ag[kMaxRanks];
  uint2* ag_mc;
  int* state;
  int rank;
  int world;
  int64_t max_pairs;  // capacity of ag (and of the world chunks of rs), in bf16 pairs
};

// out[M, N] (bf16, row stride ldd) = sum over ranks of (sum of the `splits`
// fp32 [M, N] slabs of ws on that rank).  Needs N even and M * N / 2 <= max_pairs.
void finalize_ll(const float* ws, int splits, int M, int N, __nv_bfloat16* out, int64_t ldd, const LLArgs& a,
                 cudaStream_t stream);

}  // namespace ar
}  // namespace lf
