// Memory-bound sm_100a kernels of the decoder step: embedding gather,
// RMSNorm with fused residual add, RoPE fused with the paged-KV write, SwiGLU,
// and the on-device samplers (greedy argmax and top-k / top-p / temperature).
//
// Oracle semantics (reference file:line):
//   embedding         kernels/reference/basic.mbt:3-28
//   RMSNorm           kernels/reference/basic.mbt:31-68   x * rsqrt(mean(x^2) + eps) * w
//   residual add      kernels/reference/basic.mbt:156-171
//   split-half RoPE   kernels/reference/rotary.mbt:187-243
//   SiLU-gated MLP    kernels/reference/mlp.mbt:335-369
//   greedy            sampling/greedy.mbt (max finite logit, lowest id on ties)
//   stochastic        sampling/stochastic.mbt (sort desc / lowest id, top-k,
//                     max-shifted temperature softmax, smallest nucleus with
//                     mass >= top_p * total, draw where cumulative > u * mass)
//   counter RNG       sampling/rng.mbt (splitmix-style counter_state/counter_unit)
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "elementwise.h"

namespace lf {
namespace ew {

// ---------------------------------------------------------------------------
// Embedding gather: out[t, :] = E[ids[t], :]   (bf16, 16-byte vectors)
//
// Forwarded decode tokens: with `fwd` set, row t in [fwd_first, fwd_first +
// nfwd) whose fwd[t - fwd_first] = j >= 0 takes its id from prev[j] (the
// previous step's sample, still on the device while the host plans ahead)
// and stores it back into ids[t]; j outside [0, nprev) is a bad index.
// ---------------------------------------------------------------------------
__global__ void embed_kernel(int32_t* __restrict__ ids, const uint4* __restrict__ table,
                             uint4* __restrict__ out, int T, int vec_per_row, int vocab,
                             const int32_t* __restrict__ fwd, int fwd_first, int nfwd,
                             const int32_t* __restrict__ prev, int nprev) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  int id = ids[t];
  if (fwd != nullptr && t >= fwd_first && t < fwd_first + nfwd) {
    const int j = fwd[t - fwd_first];
    if (j >= 0) {
      id = (j < nprev) ? prev[j] : -1;
      __syncthreads();                       // every thread has read ids[t] before it is replaced
      if (threadIdx.x == 0) ids[t] = id;
    }
  }
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_error(kErrBadIndex, (unsigned long long)t);
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) out[(size_t)t * vec_per_row + i] = make_uint4(0, 0, 0, 0);
    return;
  }
  for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x)
    out[(size_t)t * vec_per_row + i] = table[(size_t)id * vec_per_row + i];
}

void embed(int32_t* ids, const void* table, void* out, int T, int H, int vocab, cudaStream_t s,
           const int32_t* fwd, int fwd_first, int nfwd, const int32_t* prev, int nprev) {
  if (T <= 0) return;
  const int vpr = H / 8;
  launch_k(embed_kernel, dim3(T), dim3(128), 0, s, 1,
         ids, reinterpret_cast<const uint4*>(table), reinterpret_cast<uint4*>(out), T, vpr, vocab,
         fwd, fwd_first, nfwd, prev, nprev);
}

// ---------------------------------------------------------------------------
// RMSNorm (+ residual).  If `residual` is non-null:
//   r = x + residual;  residual = r;  out = r * rsqrt(mean(r^2) + eps) * w
// else out = x * rsqrt(mean(x^2) + eps) * w.   fp32 math, bf16 storage.
// One CTA per row, each thread owns VPT 16-byte vectors held in registers.
// Gathered form (`rows` non-null): output row i normalises input row rows[i]
// and the residual is not written back (the final norm before the LM head
// only needs the sampled rows); an index outside [0, in_rows) is a bad index.
// ---------------------------------------------------------------------------
template <int VPT>
__global__ void __launch_bounds__(128) rmsnorm_kernel(const uint4* __restrict__ x, uint4* __restrict__ residual,
                                                      const uint4* __restrict__ w, uint4* __restrict__ out,
                                                      int vec_per_row, float eps, int H,
                                                      const int32_t* __restrict__ rows, int in_rows) {
  pdl_trigger();
  // The weight does not depend on the previous kernel: load it before the
  // dependency wait (under PDL this overlaps the producer's tail) instead of
  // after the reduction, where it would be a second dependent round trip.
  uint4 wreg[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * 128;
    wreg[j] = i < vec_per_row ? w[i] : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  const size_t orow = blockIdx.x;
  size_t row = orow;
  if (rows != nullptr) {
    const int r = rows[orow];
    if (r < 0 || r >= in_rows) {
      if (threadIdx.x == 0) set_error(kErrBadIndex, (unsigned long long)orow);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int i = threadIdx.x + j * 128;
        if (i < vec_per_row) out[orow * vec_per_row + i] = make_uint4(0u, 0u, 0u, 0u);
      }
      return;
    }
    row = (size_t)r;
  }
  const bool write_residual = rows == nullptr;
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
          // The residual stream is kept in bf16, as the model's activations are.
          sb[e] = __float2bfloat16(__bfloat162float(ab[e]) + __bfloat162float(rb[e]));
          v[j][e] = __bfloat162float(sb[e]);
        }
        if (write_residual) residual[row * vec_per_row + i] = sum;
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
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * 128;
    if (i < vec_per_row) {
      const uint4 wv = wreg[j];
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 o;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) ob[e] = __float2bfloat16(v[j][e] * inv * __bfloat162float(wb[e]));
      out[orow * vec_per_row + i] = o;
    }
  }
}

void rmsnorm(const void* x, void* residual, const void* w, void* out, int T, int H, float eps, cudaStream_t s,
             const int32_t* rows, int in_rows) {
  if (T <= 0) return;
  const int vpr = H / 8;
  const int vpt = (vpr + 127) / 128;
  auto X = reinterpret_cast<const uint4*>(x);
  auto R = reinterpret_cast<uint4*>(residual);
  auto W = reinterpret_cast<const uint4*>(w);
  auto O = reinterpret_cast<uint4*>(out);
  if (vpt <= 1) launch_k(rmsnorm_kernel<1>, dim3(T), dim3(128), 0, s, 1,
         X, R, W, O, vpr, eps, H, rows, in_rows);
  else if (vpt <= 2) launch_k(rmsnorm_kernel<2>, dim3(T), dim3(128), 0, s, 1,
         X, R, W, O, vpr, eps, H, rows, in_rows);
  else if (vpt <= 4) launch_k(rmsnorm_kernel<4>, dim3(T), dim3(128), 0, s, 1,
         X, R, W, O, vpr, eps, H, rows, in_rows);
  else if (vpt <= 8) launch_k(rmsnorm_kernel<8>, dim3(T), dim3(128), 0, s, 1,
         X, R, W, O, vpr, eps, H, rows, in_rows);
  else launch_k(rmsnorm_kernel<16>, dim3(T), dim3(128), 0, s, 1,
         X, R, W, O, vpr, eps, H, rows, in_rows);
}

// ---------------------------------------------------------------------------
// RoPE + paged KV write.
// qkv: [T, (Hq + 2*Hkv) * D] bf16, rows of stride ld; Q heads, then K, then V.
// Q is rotated in place.  K is rotated and, with V, written to the paged cache
// at slot_mapping[t] (= page * PAGE + offset).  Cache layout per layer and per
// K/V: [page][kv_head][PAGE][D] (one (page, head) block is contiguous).
// cos_sin: [max_pos, D/2] float2 (cos, sin) for angle = pos / theta^(2i/D).
// A negative slot skips the write (padding rows of a captured batch).
// ---------------------------------------------------------------------------
__global__ void rope_kv_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld, const int32_t* __restrict__ positions,
                               const int32_t* __restrict__ slots, const float2* __restrict__ cos_sin,
                               __nv_bfloat16* __restrict__ kcache, __nv_bfloat16* __restrict__ vcache, int Hq,
                               int Hkv, int D, int page, int max_pos, int64_t num_slots) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int half = D / 2;
  const int pos = positions[t];
  const int slot = slots[t];
  __nv_bfloat16* row = qkv + (size_t)t * ld;
  const bool pos_ok = pos >= 0 && pos < max_pos;
  if (!pos_ok && threadIdx.x == 0) set_error(kErrBadIndex, (unsigned long long)t);
  const bool slot_ok = slot >= 0 && (int64_t)slot < num_slots;
  const int pg = slot / page, off = slot % page;
  // Rotate Q and K heads: work item = (head, i) with i < D/2.
  const int n_rot = (Hq + Hkv) * half;
  for (int w = threadIdx.x; w < n_rot; w += blockDim.x) {
    const int h = w / half, i = w % half;
    __nv_bfloat16* hp = row + h * D;
    const float x1 = __bfloat162float(hp[i]);
    const float x2 = __bfloat162float(hp[i + half]);
    float2 cs = pos_ok ? cos_sin[(size_t)pos * half + i] : make_float2(1.f, 0.f);
    const __nv_bfloat16 o1 = __float2bfloat16(x1 * cs.x - x2 * cs.y);
    const __nv_bfloat16 o2 = __float2bfloat16(x2 * cs.x + x1 * cs.y);
    if (h < Hq) {
      hp[i] = o1;
      hp[i + half] = o2;
    } else if (slot_ok) {
      const int kh = h - Hq;
      __nv_bfloat16* dst = kcache + (((size_t)pg * Hkv + kh) * page + off) * D;
      dst[i] = o1;
      dst[i + half] = o2;
    }
  }
  if (slot_ok) {
    // V heads: plain copy, 8 bf16 per thread-iteration.
    const int n_v = Hkv * D / 8;
    const uint4* vsrc = reinterpret_cast<const uint4*>(row + (Hq + Hkv) * D);
    for (int w = threadIdx.x; w < n_v; w += blockDim.x) {
      const int kh = (w * 8) / D, d = (w * 8) % D;
      uint4* dst = reinterpret_cast<uint4*>(vcache + (((size_t)pg * Hkv + kh) * page + off) * D + d);
      *dst = vsrc[w];
    }
  }
}

void rope_kv_write(void* qkv, int64_t ld, const int32_t* positions, const int32_t* slots, const void* cos_sin,
                   void* kcache, void* vcache, int T, int Hq, int Hkv, int D, int page, int max_pos,
                   int64_t num_slots, cudaStream_t s) {
  if (T <= 0) return;
  launch_k(rope_kv_kernel, dim3(T), dim3(256), 0, s, 1,
         reinterpret_cast<__nv_bfloat16*>(qkv), ld, positions, slots,
                                    reinterpret_cast<const float2*>(cos_sin), reinterpret_cast<__nv_bfloat16*>(kcache),
                                    reinterpret_cast<__nv_bfloat16*>(vcache), Hq, Hkv, D, page, max_pos, num_slots);
}

// ---------------------------------------------------------------------------
// SwiGLU over a [T, 2F] gate|up buffer (gate = first F columns): out = silu(g)*u.
// Used where the gate/up projection is not the fused tcgen05 epilogue.
// ---------------------------------------------------------------------------
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int F) {
  pdl_trigger();
  pdl_wait();
  const size_t t = blockIdx.x;
  for (int i = threadIdx.x; i < F; i += blockDim.x) {
    const float g = __bfloat162float(gu[t * 2 * F + i]);
    const float u = __bfloat162float(gu[t * 2 * F + F + i]);
    const float gs = __bfloat162float(__float2bfloat16(g / (1.f + __expf(-g))));
    out[t * F + i] = __float2bfloat16(gs * u);
  }
}

void swiglu(const void* gu, void* out, int T, int F, cudaStream_t s) {
  if (T <= 0) return;
  launch_k(swiglu_kernel, dim3(T), dim3(256), 0, s, 1,
         reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<__nv_bfloat16*>(out), F);
}

// ---------------------------------------------------------------------------
// Samplers.
// ---------------------------------------------------------------------------
// Monotone map float -> uint32 (larger float => larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Composite total order used by the reference sort: larger logit first, then
// lower token id first.  Larger composite key == earlier in sorted order.
__device__ __forceinline__ uint64_t ckey(float f, int id) {
  return ((uint64_t)fkey(f) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)id);
}

template <int NT>
__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  uint64_t r = sh[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) r = sh[i] > r ? sh[i] : r;
  return r;
}

template <int NT>
__device__ __forceinline__ double block_sum_f64(double v, double* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = 0.0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh[i];
  return r;
}

template <int NT>
__device__ __forceinline__ int block_sum_i(int v, int* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh[i];
  return r;
}

// Greedy: per row, the max finite logit, lowest id on ties.  A row with a
// non-finite logit gets status -1 in out_status[row] or, without a status
// array, records kErrNonFinite (info: the row) so the step fails closed.
template <int NT>
__global__ void __launch_bounds__(NT) argmax_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                    int32_t* __restrict__ out_tok, int32_t* __restrict__ status) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t sh[NT / 32];
  __shared__ int shi[NT / 32];
  const float* row = logits + (size_t)blockIdx.x * ld;
  uint64_t best = 0;
  int bad = 0;
  for (int i = threadIdx.x; i < V; i += NT) {
    const float v = row[i];
    if (!isfinite(v)) { bad = 1; continue; }
    const uint64_t k = ckey(v, i);
    best = k > best ? k : best;
  }
  best = block_max_u64<NT>(best, sh);
  bad = block_sum_i<NT>(bad, shi);
  if (threadIdx.x == 0) {
    out_tok[blockIdx.x] = (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    if (status) status[blockIdx.x] = bad ? -1 : 0;
    else if (bad) set_error(kErrNonFinite, blockIdx.x);
  }
}

void argmax(const float* logits, int64_t ld, int R, int V, int32_t* out, int32_t* status, cudaStream_t s) {
  if (R <= 0) return;
  launch_k(argmax_kernel<1024>, dim3(R), dim3(1024), 0, s, 1,
         logits, ld, V, out, status);
}

// Vocab-parallel greedy, step 1: per row, the composite key (logit, lowest id)
// of this rank's vocab shard, with ids offset to global vocabulary ids.
// Non-finite logits are skipped (a row with none finite yields key 0).
template <int NT>
__global__ void __launch_bounds__(NT) argmax_key_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                        int id_offset, unsigned long long* __restrict__ keys) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t sh[NT / 32];
  const float* row = logits + (size_t)blockIdx.x * ld;
  uint64_t best = 0;
  bool bad = false;
  for (int i = threadIdx.x; i < V; i += NT) {
    const float v = row[i];
    if (!isfinite(v)) { bad = true; continue; }
    const uint64_t k = ckey(v, i + id_offset);
    best = k > best ? k : best;
  }
  best = block_max_u64<NT>(best, sh);
  if (bad) set_error(kErrNonFinite, blockIdx.x);   // any thread: the word keeps the first code
  if (threadIdx.x == 0) keys[blockIdx.x] = best;
}

// Step 2 (after an all-gather of keys [ranks, R]): the winning token per row.
__global__ void keys_to_tokens_kernel(const unsigned long long* __restrict__ keys, int R, int ranks,
                                      int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  uint64_t best = 0;
  for (int k = 0; k < ranks; ++k) best = keys[(size_t)k * R + r] > best ? keys[(size_t)k * R + r] : best;
  out[r] = (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
}

void argmax_keys(const float* logits, int64_t ld, int R, int V, int id_offset, unsigned long long* keys,
                 cudaStream_t s) {
  if (R <= 0) return;
  launch_k(argmax_key_kernel<1024>, dim3(R), dim3(1024), 0, s, 1,
         logits, ld, V, id_offset, keys);
}

void keys_to_tokens(const unsigned long long* keys, int R, int ranks, int32_t* out, cudaStream_t s) {
  if (R <= 0) return;
  launch_k(keys_to_tokens_kernel, dim3((R + 127) / 128), dim3(128), 0, s, 1,
         keys, R, ranks, out);
}

// Counter-addressed uniform draw in [0, 1) with 53 random bits
// (sampling/rng.mbt counter_state / counter_unit).
__host__ __device__ inline double counter_unit(uint64_t seed, int64_t sample_index) {
  uint64_t v = seed + (uint64_t)(sample_index + 1) * 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  v = v ^ (v >> 31);
  if (v == 0) v = 0x9e3779b97f4a7c15ull;
  return (double)(v >> 11) * 1.1102230246251565e-16;
}

// Inverse of fkey.
__device__ __forceinline__ float key_value(uint64_t k) {
  const uint32_t u = (uint32_t)(k >> 32);
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

// Entry sources of the sampler.  get(i, v, k) yields entry i's logit and
// composite key (false: no entry there); bad(i) says whether entry i makes
// the row invalid (a non-finite logit).
struct RowSource {  // one full logits row: entry i is token i
  const float* row;
  int n;
  __device__ __forceinline__ bool get(int i, float& v, uint64_t& k) const {
    v = row[i];
    if (!isfinite(v)) return false;
    k = ckey(v, i);
    return true;
  }
  __device__ __forceinline__ bool bad(int i) const { return !isfinite(row[i]); }
};

// The candidate keys of every vocabulary shard for one row (see
// topk_keys_kernel): `ranks` blocks of `per` words, the last word of a block
// being the shard's status (1 ok, 2 non-finite logits), unused slots 0.
struct CandidateSource {
  const unsigned long long* keys;  // [ranks][rows][per]
  int row, rows, per, n;           // n = ranks * per
  __device__ __forceinline__ const unsigned long long* at(int i) const {
    return keys + ((size_t)(i / per) * rows + row) * per + i % per;
  }
  __device__ __forceinline__ bool get(int i, float& v, uint64_t& k) const {
    if (i % per == per - 1) return false;
    k = *at(i);
    if (k == 0) return false;
    v = key_value(k);
    return true;
  }
  __device__ __forceinline__ bool bad(int i) const { return i % per == per - 1 && *at(i) == 2; }
};

template <int NT>
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, unsigned long long* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long r = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += sh[i];
  return r;
}

// Fixed-point weight of a token: exp((v - max) / T) in units of 2^-44.  Each
// weight is at most 2^44 and a row has fewer than 2^19 entries, so every sum
// fits in 64 bits; integer sums are exact and order-independent, so every
// tensor-parallel rank draws the same token from the same logits.
constexpr float kMassScale = 17592186044416.0f;   // 2^44

// Radix selection over the composite keys, largest first: the key of the
// first entry (in descending key order, restricted to keys >= floor_key) at
// which the cumulative weight satisfies  cum >= thr  (strict = false) or
// cum > thr  (strict = true).  One byte of the 64-bit key per pass (8 passes);
// each pass builds a 256-bin histogram of the entries that match the bytes
// chosen so far.  The caller guarantees that the total weight satisfies the
// predicate, so the selected key is an existing entry's.
template <int NT, class Src, class WFn>
__device__ uint64_t select_desc(const Src& src, uint64_t floor_key, WFn wfn, unsigned long long thr, bool strict,
                                unsigned long long* hist, unsigned long long* state) {
  const int n = src.n;
  uint64_t P = 0;
  unsigned long long above = 0;
  for (int d = 7; d >= 0; --d) {
    for (int i = threadIdx.x; i < 256; i += NT) hist[i] = 0;
    __syncthreads();
    const int sh = 8 * d;
    const uint64_t hi_mask = d == 7 ? 0ull : (~0ull << (sh + 8));
    if (d >= 6) {
      // The top two key bytes (sign, exponent, leading mantissa bits) put most
      // entries into a few bins: lanes of a warp with the same bin are summed
      // by shuffles first and one of them adds the group's weight.
      const int lane = threadIdx.x & 31;
      for (int base = 0; base < n; base += NT) {
        const int i = base + threadIdx.x;
        float v;
        uint64_t k;
        int bin = 256;
        unsigned long long wv = 0;
        if (i < n && src.get(i, v, k) && k >= floor_key && (k & hi_mask) == P) {
          bin = (int)((k >> sh) & 255u);
          wv = wfn(v);
        }
        const unsigned m = __match_any_sync(0xffffffffu, bin);
        // the group's sum by the warp reduction unit: a weight is below 2^44,
        // so it is added as two 22-bit limbs (32 limbs fit in 32 bits)
        const unsigned lo = __reduce_add_sync(m, (unsigned)(wv & 0x3FFFFFull));
        const unsigned hi = __reduce_add_sync(m, (unsigned)(wv >> 22));
        const unsigned long long sum = ((unsigned long long)hi << 22) + lo;
        if (bin < 256 && __ffs(m) - 1 == lane) atomicAdd(&hist[bin], sum);
      }
    } else {
      // deeper bytes: only the few entries matching the chosen prefix remain
      for (int i = threadIdx.x; i < n; i += NT) {
        float v;
        uint64_t k;
        if (src.get(i, v, k) && k >= floor_key && (k & hi_mask) == P)
          atomicAdd(&hist[(k >> sh) & 255u], wfn(v));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long a = above;
      int b = 255;
      for (; b > 0; --b) {
        const unsigned long long c = a + hist[b];
        if (strict ? c > thr : c >= thr) break;
        a = c;
      }
      state[0] = P | ((uint64_t)b << sh);
      state[1] = a;
    }
    __syncthreads();
    P = state[0];
    above = state[1];
    __syncthreads();
  }
  return P;
}

// Counter-addressed sampling of one row (block of NT threads).  Every quantity
// over the reference's sorted order (logit descending, id ascending == the
// composite key descending) is the crossing point of a cumulative count or
// mass, found by radix selection on the 64-bit key (8 passes each): the
// k-th largest key (top-k), the first key at which the cumulative mass reaches
// top_p of the total (top-p), the first key at which it exceeds u times the
// retained mass (the draw).  About 28 passes over the row, no sort, no global
// scratch.  The result depends only on the entries' keys, so a row given as
// per-shard candidates (every key of the top-k set present) samples the same
// token as the full row.
template <int NT, class Src>
__device__ void sample_row(const Src& src, const SampleParams p, int32_t* out_tok, int32_t* status, uint64_t* shk,
                           double* shd, int* shi) {
  (void)shd;
  __shared__ unsigned long long hist[256];
  __shared__ unsigned long long state[2];
  __shared__ unsigned long long shu[NT / 32];
  const int n = src.n;
  // Pass 1: validation, the top key (max logit, lowest id), the finite count.
  uint64_t best = 0;
  int bad = 0, finite = 0;
  for (int i = threadIdx.x; i < n; i += NT) {
    float v;
    uint64_t k;
    if (src.bad(i)) bad = 1;
    if (src.get(i, v, k)) {
      best = k > best ? k : best;
      ++finite;
    }
  }
  best = block_max_u64<NT>(best, shk);
  bad = block_sum_i<NT>(bad, shi);
  finite = block_sum_i<NT>(finite, shi);
  const int top_id = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  if (bad) {
    if (threadIdx.x == 0) {
      *out_tok = top_id;
      if (status) *status = -1;
      else set_error(kErrNonFinite, blockIdx.x);
    }
    return;
  }
  if (p.mode == 0 || !(p.temperature > 0.f)) {
    if (threadIdx.x == 0) { *out_tok = top_id; if (status) *status = 0; }
    return;
  }
  const float mx = key_value(best);
  const float inv_t = 1.0f / p.temperature;
  auto one = [](float) -> unsigned long long { return 1ull; };
  auto mass = [&](float v) -> unsigned long long { return __float2ull_rn(__expf((v - mx) * inv_t) * kMassScale); };
  auto mass_ge = [&](uint64_t K) -> unsigned long long {
    unsigned long long m = 0;
    for (int i = threadIdx.x; i < n; i += NT) {
      float v;
      uint64_t k;
      if (src.get(i, v, k) && k >= K) m += mass(v);
    }
    return block_sum_u64<NT>(m, shu);
  };

  // Top-k: the k-th largest key.
  uint64_t kfloor = 0;
  if (p.top_k > 0 && finite > p.top_k) kfloor = select_desc<NT>(src, 0, one, (unsigned long long)p.top_k, false, hist, state);
  const unsigned long long total = mass_ge(kfloor);

  // Top-p: the smallest prefix whose cumulative mass reaches top_p * total.
  uint64_t pfloor = kfloor;
  unsigned long long retained = total;
  if (p.top_p > 0.f && p.top_p < 1.f) {
    unsigned long long thr = (unsigned long long)ceil((double)p.top_p * (double)total);
    if (thr < 1ull) thr = 1ull;
    pfloor = select_desc<NT>(src, kfloor, mass, thr, false, hist, state);
    retained = mass_ge(pfloor);
  }

  // Draw: the first sorted token whose inclusive cumulative mass exceeds u * retained.
  const double u = counter_unit(p.seed, p.sample_index);
  const unsigned long long target = (unsigned long long)floor(u * (double)retained);
  const uint64_t sel = select_desc<NT>(src, pfloor, mass, target, true, hist, state);
  if (threadIdx.x == 0) {
    *out_tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(sel & 0xFFFFFFFFull));
    if (status) *status = 0;
  }
}

// Per-row sampling parameters (SampleParams in elementwise.h); mode 0 =
// greedy, 1 = sample.
template <int NT>
__global__ void __launch_bounds__(NT) sample_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                    const SampleParams* __restrict__ params,
                                                    int32_t* __restrict__ out_tok, int32_t* __restrict__ status) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t shk[NT / 32];
  __shared__ double shd[NT / 32];
  __shared__ int shi[NT / 32];
  const int r = blockIdx.x;
  const RowSource src{logits + (size_t)r * ld, V};
  sample_row<NT>(src, params[r], out_tok + r, status ? status + r : nullptr, shk, shd, shi);
}

// Vocabulary-parallel sampling, step 1: per row, the keys of this shard's kc
// largest finite logits (token ids offset by id_offset) and a status word
// (1 ok, 2 the shard has non-finite logits): out[row][0..kc] (unused slots 0).
// The kc-th largest key is found by bisection on the key space.
template <int NT>
__global__ void __launch_bounds__(NT) topk_keys_kernel(const float* __restrict__ logits, int64_t ld, int V,
                                                       int id_offset, int kc,
                                                       unsigned long long* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t shk[NT / 32];
  __shared__ int shi[NT / 32];
  __shared__ int s_count;
  const float* row = logits + (size_t)blockIdx.x * ld;
  unsigned long long* dst = out + (size_t)blockIdx.x * (kc + 1);
  uint64_t best = 0;
  int bad = 0, finite = 0;
  for (int i = threadIdx.x; i < V; i += NT) {
    const float v = row[i];
    if (!isfinite(v)) { bad = 1; continue; }
    ++finite;
    const uint64_t k = ckey(v, i + id_offset);
    best = k > best ? k : best;
  }
  best = block_max_u64<NT>(best, shk);
  bad = block_sum_i<NT>(bad, shi);
  finite = block_sum_i<NT>(finite, shi);
  uint64_t thr = 0;
  if (finite > kc) {
    uint64_t lo = 0, hi = best;  // count of keys >= lo is >= kc
    while (lo < hi) {
      const uint64_t mid = lo + (hi - lo + 1) / 2;
      int c = 0;
      for (int i = threadIdx.x; i < V; i += NT) {
        const float v = row[i];
        c += isfinite(v) && ckey(v, i + id_offset) >= mid;
      }
      if (block_sum_i<NT>(c, shi) >= kc) lo = mid; else hi = mid - 1;
    }
    thr = lo;
  }
  if (threadIdx.x == 0) s_count = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += NT) {
    const float v = row[i];
    if (!isfinite(v)) continue;
    const uint64_t k = ckey(v, i + id_offset);
    if (k >= thr) {
      const int slot = atomicAdd(&s_count, 1);
      if (slot < kc) dst[slot] = k;
    }
  }
  __syncthreads();
  for (int j = s_count + threadIdx.x; j < kc; j += NT) dst[j] = 0;
  if (threadIdx.x == 0) dst[kc] = bad ? 2ull : 1ull;
}

// Vocabulary-parallel sampling, step 2: the draw over the gathered candidates
// of every shard (keys [ranks][rows][kc + 1]).  Exact when every stochastic
// row has 0 < top_k <= kc (the top-k set is then among the candidates).
template <int NT>
__global__ void __launch_bounds__(NT) sample_keys_kernel(const unsigned long long* __restrict__ keys, int rows,
                                                         int ranks, int kc, const SampleParams* __restrict__ params,
                                                         int32_t* __restrict__ out_tok, int32_t* __restrict__ status) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t shk[NT / 32];
  __shared__ double shd[NT / 32];
  __shared__ int shi[NT / 32];
  const int r = blockIdx.x;
  const CandidateSource src{keys, r, rows, kc + 1, ranks * (kc + 1)};
  sample_row<NT>(src, params[r], out_tok + r, status ? status + r : nullptr, shk, shd, shi);
}

void topk_keys(const float* logits, int64_t ld, int R, int V, int id_offset, int kc, unsigned long long* out,
               cudaStream_t s) {
  if (R <= 0) return;
  launch_k(topk_keys_kernel<512>, dim3(R), dim3(512), 0, s, 1, logits, ld, V, id_offset, kc, out);
}

void sample_keys(const unsigned long long* keys, int R, int ranks, int kc, const SampleParams* params, int32_t* out,
                 int32_t* status, cudaStream_t s) {
  if (R <= 0) return;
  launch_k(sample_keys_kernel<256>, dim3(R), dim3(256), 0, s, 1, keys, R, ranks, kc, params, out, status);
}

void sample(const float* logits, int64_t ld, int R, int V, const SampleParams* params, int32_t* out, int32_t* status,
            cudaStream_t s) {
  if (R <= 0) return;
  launch_k(sample_kernel<512>, dim3(R), dim3(512), 0, s, 1,
         logits, ld, V, params, out, status);
}

double host_counter_unit(uint64_t seed, int64_t idx) { return counter_unit(seed, idx); }

}  // namespace ew
}  // namespace lf
