// RMSNorm with the sequence-parallel all-gather in its epilogue (sp_gather.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace sp {

constexpr int kMaxRanks = 8;

struct GatherArgs {
  __nv_bfloat16* dst[kMaxRanks];          // the gathered [world * rows_local, H] buffer on each rank
  unsigned long long* flag[kMaxRanks];    // [world] arrival words on each rank (epoch, per source)
  int* state;                             // local: epoch, completion counter
  int rank, world, rows_local;
};

// out rows = RMSNorm(x (+ residual, written back)) of this rank's rows_local
// rows, stored into every rank's gathered buffer at rows [rank * rows_local, ...);
// the grid's last CTA then publishes this operation's epoch to every rank.
void norm_gather(const void* x, void* residual, const void* w, float eps, int H, const GatherArgs& g,
                 cudaStream_t s);
// Waits (bounded) for every rank's word of the current operation, then
// advances the epoch.  The consumer of the gathered rows follows on the stream.
void gather_wait(const GatherArgs& g, cudaStream_t s);

}  // namespace sp
}  // namespace lf
