// Expert-parallel dispatch and combine over NVLink peer memory.
//
// Sequence-parallel MoE layer, per rank (T local tokens, k routes each, El
// experts per rank, W ranks):
//   1. plan      stable counting sort of this rank's T * k pairs by the rank
//                that holds the pair's expert: slot of each pair in its
//                destination's receive area, pairs per destination;
//   2. dispatch  every pair's hidden row and (local expert, pair index) are
//                stored straight into the destination rank's receive area
//                (peer stores); when the whole grid is done, the last CTA
//                publishes (epoch << 32 | pairs) to every destination;
//   3. receive   one CTA waits for every source's word of this epoch, then
//      plan      lays the received rows out in expert order, each expert's
//                segment padded to 128 rows (the grouped GEMM's row blocks);
//   4. gather    the rows into the grouped GEMM's input;
//   (the grouped gate/up + SwiGLU and down GEMMs run here, unchanged)
//   5. combine   every output row goes back to its source's combine area at
//      send      its pair index (peer stores); the last CTA publishes
//                (epoch << 32 | rows) to every source;
//   6. combine   every CTA waits for every expert rank's word, then sums each
//      receive   token's k returned rows with its routing weights; the grid's
//                last CTA advances the epoch.
// No host round trip (the grouped GEMM reads its segments on the device), so
// the layer can be captured in a CUDA graph.  A rank writes a peer's receive
// area for layer l + 1 only after its combine of layer l, which needed that
// peer's returned rows, which the peer sent after its GEMMs had read layer l's
// rows; the combine area is re-used after the same chain in the other
// direction.  The words carry the epoch, so they are never reset.  Every wait
// is bounded; a timeout records kErrPeerTimeout and the kernel goes on.
//
// The reference has no expert parallelism (MoE is a v1 non-goal there:
// docs/PRODUCT_CONTRACT.md:172); this file has no counterpart.
#include <stdexcept>

#include "common.cuh"
#include "moe_a2a.h"

namespace lf {
namespace a2a {

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Waits (bounded) until the word carries epoch `ep`; returns its low half, or
// -1 after recording a timeout.
__device__ int wait_word(const unsigned long long* p, uint32_t ep, unsigned long long where) {
  unsigned long long v = ld_acquire_u64(p);
  if ((uint32_t)(v >> 32) != ep) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    do {
      if ((++spins & 255u) == 0) {
        if (error_pending()) return -1;
        if (globaltimer_ns() - t0 > wait_limit_ns()) {
          set_error(kErrPeerTimeout, where);
          return -1;
        }
      }
      v = ld_acquire_u64(p);
    } while ((uint32_t)(v >> 32) != ep);
  }
  return (int)(v & 0xFFFFFFFFull);
}

// Block-wide exclusive prefix of a 0/1 flag (blockDim.x a multiple of 32, at
// most 1024); returns the prefix and writes the block total to *total.
__device__ int block_prefix(int flag, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const unsigned m = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(m & ((1u << lane) - 1u));
  __syncthreads();
  if (lane == 0) warp_sums[warp] = __popc(m);
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < nw; ++i) {
      const int c = warp_sums[i];
      warp_sums[i] = acc;
      acc += c;
    }
    *total = acc;
  }
  __syncthreads();
  return warp_sums[warp] + in_warp;
}

// 1. plan (one CTA): slot of each pair within its destination, pairs per destination.
__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ ids, int n, int32_t* __restrict__ slot,
                                                    Args a) {
  pdl_trigger();
  pdl_wait();
  __shared__ int warp_sums[32];
  __shared__ int total;
  __shared__ int running[kMaxRanks];
  if (threadIdx.x < kMaxRanks) running[threadIdx.x] = 0;
  __syncthreads();
  for (int base = 0; base < n; base += blockDim.x) {
    const int p = base + threadIdx.x;
    int dest = -1;
    if (p < n) {
      const int e = ids[p];
      dest = e / a.experts_local;
      if (e < 0 || dest >= a.world) {
        set_error(kErrBadIndex, (unsigned long long)p);
        dest = -1;
      }
    }
    for (int d = 0; d < a.world; ++d) {
      const int pos = block_prefix(dest == d, warp_sums, &total);
      if (dest == d) slot[p] = running[d] + pos;
      __syncthreads();
      if (threadIdx.x == 0) running[d] += total;
      __syncthreads();
    }
  }
  if (threadIdx.x < a.world) a.counts[threadIdx.x] = running[threadIdx.x];
}

// 2. dispatch: rows and meta into the destinations' receive areas, then the words.
__global__ void __launch_bounds__(256) dispatch_kernel(const __nv_bfloat16* __restrict__ h,
                                                       const int32_t* __restrict__ ids, int n,
                                                       const int32_t* __restrict__ slot, Args a) {
  pdl_trigger();
  pdl_wait();
  const uint32_t ep = (uint32_t)(*reinterpret_cast<volatile int*>(a.state)) + 1u;
  const int vecs = a.hidden / 8;
  for (int p = blockIdx.x; p < n; p += gridDim.x) {
    const int e = ids[p];
    const int dest = e / a.experts_local;
    const int s = slot[p];
    if (e < 0 || dest >= a.world || s < 0 || s >= a.cap) continue;  // recorded by the plan kernel
    const uint4* src = reinterpret_cast<const uint4*>(h + (size_t)(p / a.topk) * a.hidden);
    const size_t row = (size_t)a.rank * a.cap + s;
    uint4* dst = reinterpret_cast<uint4*>(a.recv_x[dest] + row * a.hidden);
    for (int v = threadIdx.x; v < vecs; v += blockDim.x) dst[v] = src[v];
    if (threadIdx.x == 0) a.recv_meta[dest][row] = make_int2(e - dest * a.experts_local, p);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    if (atom_add_acq_rel(a.state + 1, 1) == (int)gridDim.x - 1) {
      a.state[1] = 0;
      fence_acq_rel_sys();
      for (int d = 0; d < a.world; ++d)
        st_release_u64(a.recv_flag[d] + a.rank, ((unsigned long long)ep << 32) | (unsigned)a.counts[d]);
    }
  }
}

// 3. receive plan (one CTA): wait for every source, expert-ordered layout.
__global__ void __launch_bounds__(1024) receive_plan_kernel(int32_t* __restrict__ groups, int32_t* __restrict__ perm,
                                                            long long* __restrict__ back, int rows_max, Args a) {
  pdl_trigger();
  pdl_wait();
  __shared__ int n_src[kMaxRanks];
  __shared__ int off_src[kMaxRanks + 1];
  __shared__ int cnt[256];
  __shared__ int seg[257];
  const uint32_t ep = (uint32_t)(*reinterpret_cast<volatile int*>(a.state)) + 1u;
  const int El = a.experts_local;
  if (threadIdx.x < a.world) {
    const int c = wait_word(a.recv_flag[a.rank] + threadIdx.x, ep, 0xA2A00ull + threadIdx.x);
    n_src[threadIdx.x] = (c < 0 || c > a.cap) ? 0 : c;
  }
  for (int e = threadIdx.x; e < El; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    off_src[0] = 0;
    for (int s = 0; s < a.world; ++s) {
      off_src[s + 1] = off_src[s] + n_src[s];
      a.counts[a.world + s] = n_src[s];
    }
  }
  __syncthreads();
  const int R = off_src[a.world];
  const int2* meta = a.recv_meta[a.rank];
  for (int q = threadIdx.x; q < R; q += blockDim.x) {
    int s = 0;
    while (q >= off_src[s + 1]) ++s;
    const int le = meta[(size_t)s * a.cap + (q - off_src[s])].x;
    if (le >= 0 && le < El) atomicAdd(&cnt[le], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    seg[0] = 0;
    for (int e = 0; e < El; ++e) seg[e + 1] = seg[e] + ((cnt[e] + 127) / 128) * 128;
    if (seg[El] > rows_max) {
      set_error(kErrBadIndex, 0xA2A10ull);
      for (int e = 0; e <= El; ++e) seg[e] = 0;   // nothing runs rather than out of bounds
    }
    for (int e = 0; e <= El; ++e) groups[e] = seg[e];
    for (int e = 0; e < El; ++e) cnt[e] = 0;      // becomes each segment's cursor
  }
  __syncthreads();
  for (int i = threadIdx.x; i < seg[El]; i += blockDim.x) perm[i] = -1;
  __syncthreads();
  if (seg[El] == 0) return;
  for (int q = threadIdx.x; q < R; q += blockDim.x) {
    int s = 0;
    while (q >= off_src[s + 1]) ++s;
    const int j = q - off_src[s];
    const int2 m = meta[(size_t)s * a.cap + j];
    if (m.x < 0 || m.x >= El) continue;
    const int pos = seg[m.x] + atomicAdd(&cnt[m.x], 1);
    perm[pos] = s * a.cap + j;
    back[pos] = ((long long)s << 32) | (unsigned)m.y;
  }
}

// 4. gather: x[row] = received row perm[row] (zeros for padding rows).
__global__ void __launch_bounds__(256) gather_kernel(const int32_t* __restrict__ groups,
                                                     const int32_t* __restrict__ perm, __nv_bfloat16* __restrict__ x,
                                                     Args a) {
  pdl_trigger();
  pdl_wait();
  const int rows = groups[a.experts_local];
  const int vecs = a.hidden / 8;
  const uint4* recv = reinterpret_cast<const uint4*>(a.recv_x[a.rank]);
  uint4* dst = reinterpret_cast<uint4*>(x);
  const long long total = (long long)rows * vecs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / vecs), v = (int)(i % vecs);
    const int src = perm[r];
    dst[i] = src >= 0 ? recv[(size_t)src * vecs + v] : make_uint4(0, 0, 0, 0);
  }
}

// 5. combine send: output rows back to their sources, then the words.
__global__ void __launch_bounds__(256) combine_send_kernel(const __nv_bfloat16* __restrict__ y,
                                                           const int32_t* __restrict__ groups,
                                                           const int32_t* __restrict__ perm,
                                                           const long long* __restrict__ back, Args a) {
  pdl_trigger();
  pdl_wait();
  const uint32_t ep = (uint32_t)(*reinterpret_cast<volatile int*>(a.state)) + 1u;
  const int rows = groups[a.experts_local];
  const int vecs = a.hidden / 8;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    if (perm[r] < 0) continue;
    const int s = (int)(back[r] >> 32);
    const int p = (int)(back[r] & 0xFFFFFFFFll);
    if (s < 0 || s >= a.world || p < 0 || p >= a.cap) continue;
    const uint4* src = reinterpret_cast<const uint4*>(y + (size_t)r * a.hidden);
    uint4* dst = reinterpret_cast<uint4*>(a.comb_y[s] + (size_t)p * a.hidden);
    for (int v = threadIdx.x; v < vecs; v += blockDim.x) dst[v] = src[v];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    if (atom_add_acq_rel(a.state + 2, 1) == (int)gridDim.x - 1) {
      a.state[2] = 0;
      fence_acq_rel_sys();
      for (int s = 0; s < a.world; ++s)
        st_release_u64(a.comb_flag[s] + a.rank, ((unsigned long long)ep << 32) | (unsigned)a.counts[a.world + s]);
    }
  }
}

// 6. combine receive: wait for every expert rank, weighted sum, advance the epoch.
__global__ void __launch_bounds__(256) combine_receive_kernel(const float* __restrict__ w, int T,
                                                              __nv_bfloat16* __restrict__ out, Args a) {
  pdl_trigger();
  pdl_wait();
  const uint32_t ep = (uint32_t)(*reinterpret_cast<volatile int*>(a.state)) + 1u;
  if (threadIdx.x < a.world) wait_word(a.comb_flag[a.rank] + threadIdx.x, ep, 0xA2A20ull + threadIdx.x);
  __syncthreads();
  const __nv_bfloat16* comb = a.comb_y[a.rank];
  const int H = a.hidden, k = a.topk;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2) {
      float2 acc = make_float2(0.f, 0.f);
      for (int j = 0; j < k; ++j) {
        const float wt = w[(size_t)t * k + j];
        const float2 v = __bfloat1622float2(
            *reinterpret_cast<const __nv_bfloat162*>(comb + ((size_t)t * k + j) * H + c));
        acc.x += wt * v.x;
        acc.y += wt * v.y;
      }
      *reinterpret_cast<__nv_bfloat162*>(out + (size_t)t * H + c) = __floats2bfloat162_rn(acc.x, acc.y);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && atom_add_acq_rel(a.state + 3, 1) == (int)gridDim.x - 1) {
    a.state[3] = 0;
    *reinterpret_cast<volatile int*>(a.state) = (int)ep;
  }
}

// ---------------------------------------------------------------------------
static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

static void check(const Args& a) {
  if (a.world < 1 || a.world > kMaxRanks || a.rank < 0 || a.rank >= a.world || a.hidden % 8 != 0 ||
      a.experts_local < 1 || a.experts_local > 256 || a.topk < 1 || a.cap < 1)
    throw std::runtime_error("lunaflux moe all-to-all: bad arguments");
}

void dispatch(const __nv_bfloat16* h, const int32_t* ids, int T, int32_t* slot, const Args& a, cudaStream_t s) {
  check(a);
  const int n = T * a.topk;
  if (n > a.cap) throw std::runtime_error("lunaflux moe all-to-all: more pairs than the receive capacity");
  launch_k(plan_kernel, dim3(1), dim3(1024), 0, s, 1, ids, n, slot, a);
  // the grid is one wave: every CTA counts itself into the completion counter
  int grid = n < 4 * sm_count() ? n : 4 * sm_count();
  if (grid < 1) grid = 1;
  launch_k(dispatch_kernel, dim3(grid), dim3(256), 0, s, 1, h, ids, n, static_cast<const int32_t*>(slot), a);
}

void receive_plan(int32_t* groups, int32_t* perm, long long* back, int rows_max, const Args& a, cudaStream_t s) {
  check(a);
  launch_k(receive_plan_kernel, dim3(1), dim3(1024), 0, s, 1, groups, perm, back, rows_max, a);
}

void gather(const int32_t* groups, const int32_t* perm, __nv_bfloat16* x, int rows_max, const Args& a,
            cudaStream_t s) {
  check(a);
  (void)rows_max;
  launch_k(gather_kernel, dim3(2 * sm_count()), dim3(256), 0, s, 1, groups, perm, x, a);
}

void combine_send(const __nv_bfloat16* y, const int32_t* groups, const int32_t* perm, const long long* back,
                  const Args& a, cudaStream_t s) {
  check(a);
  launch_k(combine_send_kernel, dim3(2 * sm_count()), dim3(256), 0, s, 1, y, groups, perm, back, a);
}

void combine_receive(const float* w, int T, __nv_bfloat16* out, const Args& a, cudaStream_t s) {
  check(a);
  int grid = T < 2 * sm_count() ? T : 2 * sm_count();
  if (grid < 1) grid = 1;
  launch_k(combine_receive_kernel, dim3(grid), dim3(256), 0, s, 1, w, T, out, a);
}

}  // namespace a2a
}  // namespace lf
