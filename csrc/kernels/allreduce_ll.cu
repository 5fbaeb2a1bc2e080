// Low-latency two-step all-reduce over NVLink peer memory, fused with the
// split-K finalisation of the row-parallel decode GEMMs.
//
// A decode step's o_proj / down output is small (a few MB), so the all-reduce
// is bound by latency, not bandwidth.  A flag-and-fence protocol pays a
// system-scope release (a fence that waits for every earlier store to be
// acknowledged) and a remote round trip per synchronisation point, twice.
// Here every 8-byte word carries two bf16 values and the epoch of the
// operation, written by one store; a reader polls its own (local) inbox until
// the epoch matches and then holds the data.  No fence, no flag, no barrier:
// the critical path is two one-way NVLink latencies.
//
//   1. reduce-scatter: each rank sums its split-K slabs for every bf16 pair
//      and stores the partial into the inbox of the pair's owner rank (pairs
//      are dealt to the ranks in contiguous chunks);
//   2. the owner polls its inbox for the other ranks' partials, adds its own,
//      writes the result and stores it (with the epoch) into every rank's
//      all-gather inbox (one multicast store through the NVSwitch, or one
//      store per peer);
//   3. every rank polls its all-gather inbox for the pairs it does not own.
//
// Inboxes are reused by consecutive operations without a barrier: a rank
// only writes a peer's inbox for operation k+1 after receiving that peer's
// contribution to k+1, which the peer sends only after finishing operation k.
// The epoch lives in device memory and is advanced by the last CTA to finish,
// so CUDA-graph replays continue the sequence.  Every wait is bounded.
//
// Traffic per rank: 2 x 8 bytes x (world - 1) / world per output pair each
// way, twice the bf16 payload (the price of the in-word epoch).
//
// The reference has no collective layer (NCCL is a planned private ABI:
// docs/PLAN.md:686, docs/ARCHITECTURE.md:451); this kernel has no counterpart.
#include <stdexcept>

#include "allreduce_ll.h"
#include "common.cuh"
#include "ll_words.cuh"

namespace lf {
namespace ar {

__device__ __forceinline__ float2 slab_pair(const float* __restrict__ ws, size_t slab, int splits, int64_t p) {
  float2 acc = make_float2(0.f, 0.f);
  for (int s = 0; s < splits; ++s) {
    const float2 v = *reinterpret_cast<const float2*>(ws + s * slab + 2 * p);
    acc.x += v.x;
    acc.y += v.y;
  }
  return acc;
}

__global__ void __launch_bounds__(256, 2) finalize_ll_kernel(const float* __restrict__ ws, int splits, int M, int N,
                                                             __nv_bfloat16* __restrict__ out, int64_t ldd,
                                                             LLArgs a) {
  pdl_trigger();
  pdl_wait();
  const int64_t half = N / 2;
  const int64_t P = (int64_t)M * half;
  const int64_t chunk = (P + a.world - 1) / a.world;
  const size_t slab = (size_t)M * N;
  const uint32_t ep = (uint32_t)(*reinterpret_cast<volatile int*>(a.state)) + 1u;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t p0 = a.rank * chunk;
  const int64_t p1 = p0 + chunk < P ? p0 + chunk : P;
  auto out_word = [&](int64_t p) {
    return reinterpret_cast<uint32_t*>(out + (p / half) * ldd + 2 * (p % half));
  };

  // 1. reduce-scatter: partials of the pairs other ranks own
  for (int64_t p = first; p < P; p += stride) {
    const int owner = (int)(p / chunk);
    if (owner == a.rank) continue;
    const float2 v = slab_pair(ws, slab, splits, p);
    st_word(a.rs[owner] + (int64_t)a.rank * chunk + (p - owner * chunk), pack2(v.x, v.y), ep);
  }
  // 2. this rank's pairs: sum, write, all-gather
  bool ok = true;
  for (int64_t p = p0 + first; p < p1 && ok; p += stride) {
    float2 acc = slab_pair(ws, slab, splits, p);
    // the same bf16 rounding of every rank's partial
    acc = unpack2(pack2(acc.x, acc.y));
    for (int src = 0; src < a.world; ++src) {
      if (src == a.rank) continue;
      uint32_t d;
      if (!poll_word(a.rs[a.rank] + (int64_t)src * chunk + (p - p0), ep, &d)) {
        ok = false;
        break;
      }
      const float2 v = unpack2(d);
      acc.x += v.x;
      acc.y += v.y;
    }
    const uint32_t r = pack2(acc.x, acc.y);
    *out_word(p) = r;
    if (a.ag_mc != nullptr) {
      st_word_mc(a.ag_mc + p, r, ep);   // every rank's inbox, this one included
    } else {
      for (int k = 0; k < a.world; ++k)
        if (k != a.rank) st_word(a.ag[k] + p, r, ep);
    }
  }
  // 3. the pairs other ranks own
  for (int64_t p = first; p < P && ok; p += stride) {
    if (p >= p0 && p < p1) continue;
    uint32_t d;
    if (!poll_word(a.ag[a.rank] + p, ep, &d)) break;
    *out_word(p) = d;
  }
  // advance the epoch once every CTA has read it
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(a.state + 1, 1) == (int)gridDim.x - 1) {
      a.state[1] = 0;
      *reinterpret_cast<volatile int*>(a.state) = (int)ep;
    }
  }
}

void finalize_ll(const float* ws, int splits, int M, int N, __nv_bfloat16* out, int64_t ldd, const LLArgs& a,
                 cudaStream_t stream) {
  if (M <= 0) return;
  if (N % 2 != 0 || (int64_t)M * N / 2 > a.max_pairs) throw std::runtime_error("lunaflux finalize_ll: shape");
  if (a.world < 1 || a.world > kMaxRanks || a.rank < 0 || a.rank >= a.world)
    throw std::runtime_error("lunaflux finalize_ll: rank");
  // Every CTA must be resident (a CTA may wait for data that a peer's CTA
  // only sends after its own waits), and the grid only has to be big enough
  // to keep enough stores in flight.
  static int per_sm = 0, sms = 0;
  if (per_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, finalize_ll_kernel, 256, 0);
    if (per_sm < 1) throw std::runtime_error("lunaflux finalize_ll: kernel cannot be resident");
    if (per_sm > 2) per_sm = 2;
  }
  const int64_t pairs = (int64_t)M * N / 2;
  const int64_t want = (pairs / a.world + 255) / 256;
  const int cap = per_sm * sms;
  const int grid = (int)(want < 1 ? 1 : (want < cap ? want : cap));
  launch_k(finalize_ll_kernel, dim3(grid), dim3(256), 0, stream, 1,
         ws, splits, M, N, out, ldd, a);
}

}  // namespace ar
}  // namespace lf
