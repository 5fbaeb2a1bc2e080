// Mixture-of-experts kernels for sm_100a (Mixtral-style top-k routing).
//
// Oracle: Mixtral's sparse MoE block — softmax over the router logits, keep
// the top-k experts, renormalise their weights, y = sum_k w_k * Expert_k(x)
// with Expert = SwiGLU MLP.  The reference has no MoE (deferred:
// docs/PLAN.md:779-790); this is new for the B200 build.
//
// Pipeline per layer (all device-side, graph-capturable, no host sync):
//   moe_route   one warp per token: router logits (fp32), softmax, top-k,
//               renormalised weights (optional per-expert logit bias for
//               load-skew experiments)
//   moe_align   one CTA: per-expert counts of this rank's experts, segment
//               offsets padded to 128 rows (a GEMM row block never straddles
//               two experts), the row -> token permutation and the
//               (token, k) -> row slots
//   moe_gather  copies token rows into expert order (padding rows zero)
//   grouped tcgen05 GEMMs (gate/up + SwiGLU, then down) over the segments
//   moe_combine y[t] = sum_k w[t,k] * expert_out[slot[t,k]] over local experts
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "moe.h"

namespace lf {
namespace moe {

constexpr int kMaxExperts = 64;
constexpr int kMaxTopK = 8;

// One CTA of kRouteThreads per token: each thread takes every 128th group of
// 8 hidden features, the per-expert partial logits are reduced through shared
// memory, and thread 0 does the softmax and the top-k (ties: lowest expert id).
constexpr int kRouteThreads = 128;

template <int E>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const __nv_bfloat16* __restrict__ h,
                                                              const float* __restrict__ wr,
                                                              const float* __restrict__ bias, int T, int H, int topk,
                                                              int32_t* __restrict__ ids, float* __restrict__ weights) {
  pdl_trigger();
  pdl_wait();
  __shared__ float part[kRouteThreads / 32][E];
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const __nv_bfloat16* x = h + (size_t)t * H;
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += kRouteThreads * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(x + i);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
    float xf[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) xf[j] = __bfloat162float(b[j]);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float4 w0 = *reinterpret_cast<const float4*>(wr + (size_t)e * H + i);
      const float4 w1 = *reinterpret_cast<const float4*>(wr + (size_t)e * H + i + 4);
      acc[e] += xf[0] * w0.x + xf[1] * w0.y + xf[2] * w0.z + xf[3] * w0.w + xf[4] * w1.x + xf[5] * w1.y +
                xf[6] * w1.z + xf[7] * w1.w;
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    acc[e] = warp_sum(acc[e]);
    if (lane == 0) part[warp][e] = acc[e];
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  float logit[E];
  float mx = -INFINITY;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kRouteThreads / 32; ++w) a += part[w][e];
    if (bias != nullptr) a += bias[e];
    logit[e] = a;
    mx = fmaxf(mx, a);
  }
  float p[E];
#pragma unroll
  for (int e = 0; e < E; ++e) p[e] = __expf(logit[e] - mx);
  // top-k by probability (ties: lowest expert id), renormalised over the k kept
  int sel[kMaxTopK];
  float ws = 0.f;
  for (int k = 0; k < topk; ++k) {
    int best = -1;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      bool taken = false;
      for (int j = 0; j < k; ++j) taken |= (sel[j] == e);
      if (!taken && (best < 0 || p[e] > p[best])) best = e;
    }
    sel[k] = best;
    ws += p[best];
  }
  for (int k = 0; k < topk; ++k) {
    ids[(size_t)t * topk + k] = sel[k];
    weights[(size_t)t * topk + k] = p[sel[k]] / ws;
  }
}

void route(const void* h, const float* wr, const float* bias, int T, int H, int E, int topk, int32_t* ids,
           float* weights, cudaStream_t s) {
  if (T <= 0) return;
  auto hp = reinterpret_cast<const __nv_bfloat16*>(h);
  const dim3 grid(T), block(kRouteThreads);
  switch (E) {
    case 2: launch_k(route_kernel<2>, grid, block, 0, s, 1, hp, wr, bias, T, H, topk, ids, weights); break;
    case 4: launch_k(route_kernel<4>, grid, block, 0, s, 1, hp, wr, bias, T, H, topk, ids, weights); break;
    case 8: launch_k(route_kernel<8>, grid, block, 0, s, 1, hp, wr, bias, T, H, topk, ids, weights); break;
    case 16: launch_k(route_kernel<16>, grid, block, 0, s, 1, hp, wr, bias, T, H, topk, ids, weights); break;
    default: break;
  }
}

// One CTA.  Local experts are [e0, e0 + El).  groups[El + 1] gets the segment
// offsets, each segment padded to a multiple of `align` rows (128, or 256 for
// the CTA-pair grouped GEMM), perm[row] the (token * topk + k) assignment of each row
// (-1 for padding), slot[t * topk + k] the row of an assignment (-1 when the
// expert is not on this rank).
__global__ void __launch_bounds__(1024) align_kernel(const int32_t* __restrict__ ids, int T, int topk, int e0,
                                                     int El, int max_rows, int align, int32_t* __restrict__ groups,
                                                     int32_t* __restrict__ perm, int32_t* __restrict__ slot) {
  __shared__ int cnt[kMaxExperts];
  __shared__ int off[kMaxExperts + 1];
  __shared__ int cursor[kMaxExperts];
  const int n = T * topk;
  for (int e = threadIdx.x; e < El; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i] - e0;
    if (e >= 0 && e < El) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < El; ++e) {
      off[e] = o;
      cursor[e] = o;
      o += (cnt[e] + align - 1) / align * align;
    }
    off[El] = o;
    if (o > max_rows) set_error(kErrBadIndex, (unsigned long long)o);
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= El; e += blockDim.x) groups[e] = min(off[e], max_rows);
  for (int r = threadIdx.x; r < max_rows; r += blockDim.x) perm[r] = -1;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i] - e0;
    int pos = -1;
    if (e >= 0 && e < El) {
      pos = atomicAdd(&cursor[e], 1);
      if (pos < max_rows) perm[pos] = i;
      else pos = -1;
    }
    slot[i] = pos;
  }
}

void align(const int32_t* ids, int T, int topk, int e0, int El, int max_rows, int32_t* groups, int32_t* perm,
           int32_t* slot, cudaStream_t s, int align_rows) {
  align_kernel<<<1, 1024, 0, s>>>(ids, T, topk, e0, El, max_rows, align_rows, groups, perm, slot);
}

__global__ void gather_kernel(const uint4* __restrict__ h, const int32_t* __restrict__ perm,
                              const int32_t* __restrict__ groups, int El, int topk, int vpr, uint4* __restrict__ out) {
  const int r = blockIdx.x;
  if (r >= groups[El]) return;
  const int a = perm[r];
  for (int i = threadIdx.x; i < vpr; i += blockDim.x)
    out[(size_t)r * vpr + i] = a < 0 ? make_uint4(0, 0, 0, 0) : h[(size_t)(a / topk) * vpr + i];
}

void gather(const void* h, const int32_t* perm, const int32_t* groups, int El, int topk, int H, int max_rows, void* out,
            cudaStream_t s) {
  gather_kernel<<<max_rows, 128, 0, s>>>(reinterpret_cast<const uint4*>(h), perm, groups, El, topk, H / 8,
                                         reinterpret_cast<uint4*>(out));
}

__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ slot,
                               const float* __restrict__ w, int topk, int H, __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < topk; ++k) {
      const int r = slot[(size_t)t * topk + k];
      if (r < 0) continue;
      const float wk = w[(size_t)t * topk + k];
      const uint4 v = *reinterpret_cast<const uint4*>(y + (size_t)r * H + i);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += wk * __bfloat162float(b[j]);
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * H + i) = make_uint4(
        pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
        pack_bf16x2(acc[6], acc[7]));
  }
}

void combine(const void* y, const int32_t* slot, const float* w, int T, int topk, int H, void* out, cudaStream_t s) {
  if (T <= 0) return;
  combine_kernel<<<T, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(y), slot, w, topk, H,
                                   reinterpret_cast<__nv_bfloat16*>(out));
}

}  // namespace moe
}  // namespace lf
