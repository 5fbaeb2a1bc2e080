// Sequence parallelism: RMSNorm (+ residual) of this rank's token rows with
// the all-gather fused into its epilogue.
//
// Each CTA normalises one local row and stores the bf16 result straight into
// every rank's gathered buffer (peer stores), at the row the token has in the
// full step; when the whole grid is done, its last CTA publishes the
// operation's epoch in every rank's arrival words.  A one-CTA wait kernel then
// holds the stream until every rank's word has arrived, so the next
// column-parallel GEMM (QKV or gate/up) reads the gathered rows from local
// memory with its own TMA loads.  No library collective and no host sync; the
// epoch lives in device memory, so graph replays continue the sequence.
//
// The caller alternates two gathered buffers over the layers of a step (a
// third one for the final norm): a rank stores into a peer's buffer for
// operation j + 2 only after the wait of operation j + 1 saw that peer's
// store of j + 1, which the peer issued after the consumer of operation j had
// run on its stream.
//
// The reference has no tensor or sequence parallelism (docs/PLAN.md:676-703);
// this file has no counterpart.
#include <stdexcept>

#include "common.cuh"
#include "sp_gather.h"

namespace lf {
namespace sp {

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Same math as the RMSNorm kernel (elementwise.cu): residual stream in bf16,
// fp32 statistics, bf16 output.
template <int VPT>
__global__ void __launch_bounds__(128) norm_gather_kernel(const uint4* __restrict__ x, uint4* __restrict__ residual,
                                                          const uint4* __restrict__ w, int vec_per_row, float eps,
                                                          int H, GatherArgs g) {
  pdl_trigger();
  pdl_wait();
  const uint32_t ep = (uint32_t)(*reinterpret_cast<volatile int*>(g.state)) + 1u;
  const size_t row = blockIdx.x;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * 128;
    if (i < vec_per_row) {
      uint4 a = x[row * vec_per_row + i];
      const __nv_bfloat16* ab = reinterpret_cast<const __nv_bfloat16*>(&a);
      if (residual != nullptr) {
        uint4 r = residual[row * vec_per_row + i];
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&r);
        uint4 sum;
        __nv_bfloat16* sb = reinterpret_cast<__nv_bfloat16*>(&sum);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          sb[e] = __float2bfloat16(__bfloat162float(ab[e]) + __bfloat162float(rb[e]));
          v[j][e] = __bfloat162float(sb[e]);
        }
        residual[row * vec_per_row + i] = sum;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j][e] = __bfloat162float(ab[e]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
    }
  }
  __shared__ float red[4];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float total = red[0] + red[1] + red[2] + red[3];
  const float inv = rsqrtf(total / (float)H + eps);
  const size_t grow = (size_t)g.rank * g.rows_local + row;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * 128;
    if (i < vec_per_row) {
      uint4 wv = w[i];
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 o;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) ob[e] = __float2bfloat16(v[j][e] * inv * __bfloat162float(wb[e]));
      for (int d = 0; d < g.world; ++d) reinterpret_cast<uint4*>(g.dst[d])[grow * vec_per_row + i] = o;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(g.state + 1) : "memory");
    if (old == (int)gridDim.x - 1) {
      g.state[1] = 0;
      fence_acq_rel_sys();
      for (int d = 0; d < g.world; ++d) st_release_u64(g.flag[d] + g.rank, (unsigned long long)ep);
    }
  }
}

__global__ void __launch_bounds__(32) gather_wait_kernel(GatherArgs g) {
  pdl_trigger();
  pdl_wait();
  const uint32_t ep = (uint32_t)(*reinterpret_cast<volatile int*>(g.state)) + 1u;
  if ((int)threadIdx.x < g.world) {
    const unsigned long long* p = g.flag[g.rank] + threadIdx.x;
    if (ld_acquire_u64(p) < ep) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_u64(p) < ep) {
        if ((++spins & 255u) == 0) {
          if (error_pending()) break;
          if (globaltimer_ns() - t0 > wait_limit_ns()) {
            set_error(kErrPeerTimeout, 0x5A900ull + threadIdx.x);
            break;
          }
        }
      }
    }
  }
  __syncwarp();
  if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(g.state) = (int)ep;
}

static void check(const GatherArgs& g, int H) {
  if (g.world < 1 || g.world > kMaxRanks || g.rank < 0 || g.rank >= g.world || g.rows_local < 0 || H % 8 != 0)
    throw std::runtime_error("lunaflux norm_gather: bad arguments");
}

void norm_gather(const void* x, void* residual, const void* w, float eps, int H, const GatherArgs& g,
                 cudaStream_t s) {
  check(g, H);
  if (g.rows_local <= 0) throw std::runtime_error("lunaflux norm_gather: no rows");
  const int vpr = H / 8;
  const int vpt = (vpr + 127) / 128;
  auto X = reinterpret_cast<const uint4*>(x);
  auto R = reinterpret_cast<uint4*>(residual);
  auto W = reinterpret_cast<const uint4*>(w);
  const dim3 grid(g.rows_local), block(128);
  if (vpt <= 1) launch_k(norm_gather_kernel<1>, grid, block, 0, s, 1, X, R, W, vpr, eps, H, g);
  else if (vpt <= 2) launch_k(norm_gather_kernel<2>, grid, block, 0, s, 1, X, R, W, vpr, eps, H, g);
  else if (vpt <= 4) launch_k(norm_gather_kernel<4>, grid, block, 0, s, 1, X, R, W, vpr, eps, H, g);
  else if (vpt <= 8) launch_k(norm_gather_kernel<8>, grid, block, 0, s, 1, X, R, W, vpr, eps, H, g);
  else launch_k(norm_gather_kernel<16>, grid, block, 0, s, 1, X, R, W, vpr, eps, H, g);
}

void gather_wait(const GatherArgs& g, cudaStream_t s) {
  check(g, 8);
  launch_k(gather_wait_kernel, dim3(1), dim3(32), 0, s, 1, g);
}

}  // namespace sp
}  // namespace lf
