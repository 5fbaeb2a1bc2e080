// Device code of the tcgen05 bf16 GEMM: the persistent warp-specialised
// kernel and the split-K finalize kernel (see gemm_bf16.cu for the design).
// Shared by the host launchers in gemm_bf16.cu and gemm_noalloc.cu.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_bf16.h"

namespace lf {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;                 // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

enum Epi : int { kStoreBf16 = 0, kStoreF32 = 1, kSwiGLU = 2, kSplitF32 = 3, kAllReduceBf16 = 4 };

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Publishes "this rank's piece with index `idx` is in its buffer" to every
// rank: one multicast reduction (NVSwitch fans it out) or one remote atomic
// per rank.  Caller has ordered its data stores before this (bar + fence).
__device__ __forceinline__ void ar_signal(const ArArgs& ar, int idx) {
  if (ar.cnt_mc != nullptr) {
    asm volatile("multimem.red.release.sys.global.add.s32 [%0], 1;" ::"l"(ar.cnt_mc + idx) : "memory");
  } else {
    for (int r = 0; r < ar.world; ++r)
      asm volatile("red.release.sys.global.add.s32 [%0], 1;" ::"l"(ar.cnt_peer[r] + idx) : "memory");
  }
}

// Waits (bounded) until every rank published piece `idx`, then re-arms the
// counter.  Returns false after recording kErrPeerTimeout.
__device__ __forceinline__ bool ar_wait(const ArArgs& ar, int idx) {
  int* c = ar.cnt_local + idx;
  if (ld_acquire_sys(c) < ar.world) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys(c) < ar.world) {
      if ((++spins & 63u) == 0) {
        if (error_pending()) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          set_error(kErrPeerTimeout, (unsigned long long)idx);
          return false;
        }
      }
    }
  }
  // Every rank has arrived; nobody signals this slot again until this rank's
  // next operation on the other slot has completed, so a plain reset is safe.
  atomicSub(c, ar.world);
  return true;
}

// Sum over ranks of 8 bf16 at element offset `off` of the slot (fp32 accumulation).
__device__ __forceinline__ uint4 ar_load_sum8(const ArArgs& ar, size_t off) {
  uint4 r;
  if (ar.mc != nullptr) {
    asm volatile("multimem.ld_reduce.weak.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(ar.mc + off)
                 : "memory");
    return r;
  }
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int k = 0; k < ar.world; ++k) {
    uint4 v;
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(ar.peer[k] + off)
                 : "memory");
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += __bfloat162float(b[e]);
  }
  return make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                    pack_bf16x2(acc[6], acc[7]));
}

template <int BN, int STAGES>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTotal = STAGES * kStageBytes + 1024 /*align slack*/ + 256 /*barriers*/;
};

template <int BN>
constexpr uint32_t tmem_cols() {
  return (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64 : (2 * BN) <= 128 ? 128 : (2 * BN) <= 256 ? 256 : 512;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

// Grouped GEMM: row block m0 -> its segment (-1 when past the used rows).
__device__ __forceinline__ int group_of(const int* groups, int num_groups, int m0) {
  if (m0 >= groups[num_groups]) return -1;
  int g = 0;
  while (g + 1 < num_groups && groups[g + 1] <= m0) ++g;
  return g;
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b, void* __restrict__ out, int M,
                     int N, int K, int ldd, int splits, int kb_per_split, ArArgs ar,
                     const int* __restrict__ groups, int num_groups) {
  // Grouped mode (groups != nullptr, mixture-of-experts): A's rows are split
  // into num_groups segments, groups[g]..groups[g+1] (each a multiple of BM,
  // read from device memory), and segment g multiplies B rows [g*N, (g+1)*N).
  // M is then an upper bound on groups[num_groups]; blocks past it are skipped.
  using S = Smem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles * splits;
  const int num_kb = (K + BK - 1) / BK;
  constexpr uint32_t kCols = tmem_cols<BN>();

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  __shared__ volatile int s_ar_ok;  // fused all-reduce: did the wait succeed

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_b = l2_policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x) {
        const int tile = unit % num_tiles;
        const int kb0 = (unit / num_tiles) * kb_per_split;
        const int kb1 = min(num_kb, kb0 + kb_per_split);
        const int m0 = (tile % num_m) * BM;
        const int n0 = (tile / num_m) * BN;
        int brow = n0;
        if (groups != nullptr) {
          const int g = group_of(groups, num_groups, m0);
          if (g < 0) continue;
          brow = g * N + n0;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, 1)) { ok = false; break; }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full_bar[stage], S::kStageBytes);
          tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * BK, m0);
          tma_load_2d_hint(sb, &tmap_b, &full_bar[stage], kb * BK, brow, pol_b);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x, ++local) {
        const int kb0 = (unit / num_tiles) * kb_per_split;
        const int kb1 = min(num_kb, kb0 + kb_per_split);
        if (groups != nullptr && group_of(groups, num_groups, ((unit % num_tiles) % num_m) * BM) < 0) {
          --local;  // skipped units use no accumulator
          continue;
        }
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            umma_f16_ss(d_tmem, sw128_kmajor_desc(sa + kk * 32), sw128_kmajor_desc(sb + kk * 32),
                        idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
    }
  } else {
    // Epilogue warps 2..5 -> TMEM lane quadrant (warp % 4).
    const int quad = warp & 3;
    int local = 0;
    for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x, ++local) {
      const int tile = unit % num_tiles;
      if (groups != nullptr && group_of(groups, num_groups, (tile % num_m) * BM) < 0) {
        --local;
        continue;
      }
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, 4)) break;
      tc_fence_after();
      const int m0 = (tile % num_m) * BM;
      const int n0 = (tile / num_m) * BN;
      const int row = m0 + quad * 32 + lane;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      if constexpr (EPI == kSwiGLU) {
        // Weight rows are interleaved in groups of 64: 32 gate rows then the
        // 32 up rows of the same output features.
        const int o0 = n0 / 2;
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 16) {
          const int grp = c / 32, off = c % 32;
          uint32_t g[16], u[16];
          tmem_ld_32x32b_x16(taddr + grp * 64 + off, g);
          tmem_ld_32x32b_x16(taddr + grp * 64 + 32 + off, u);
          tmem_wait_ld();
          if (row < M) {
            uint32_t packed[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float g0 = __uint_as_float(g[2 * j]), g1 = __uint_as_float(g[2 * j + 1]);
              const float u0 = __uint_as_float(u[2 * j]), u1 = __uint_as_float(u[2 * j + 1]);
              packed[j] = pack_bf16x2(silu(g0) * u0, silu(g1) * u1);
            }
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + o0 + c;
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c, r);
          tmem_wait_ld();
          if (row < M) {
            if constexpr (EPI == kStoreF32) {
              float* dst = reinterpret_cast<float*>(out) + (size_t)row * ldd + n0 + c;
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 8; ++j) d4[j] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            } else if constexpr (EPI == kSplitF32) {
              // Split-K partial: plain fp32 stores into this split's slab of
              // the workspace; the finalize kernel sums the slabs in a fixed
              // order, so results are bitwise reproducible.
              float* dst = reinterpret_cast<float*>(out) + (size_t)(unit / num_tiles) * M * N +
                           (size_t)row * ldd + n0 + c;
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 8; ++j) d4[j] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            } else {
              uint32_t packed[16];
#pragma unroll
              for (int j = 0; j < 16; ++j)
                packed[j] = pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
              // kAllReduceBf16 first publishes the partial tile in this rank's
              // symmetric slot (row stride N); the reduced tile goes to `out` below.
              __nv_bfloat16* dst = EPI == kAllReduceBf16
                                       ? ar.local + (size_t)row * N + n0 + c
                                       : reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + n0 + c;
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);  // the MMA warp may start the next tile now
      if constexpr (EPI == kAllReduceBf16) {
        // Tile-level all-reduce: publish, wait for the same tile of every
        // rank, then read the sum through the NVLink fabric while the MMA warp
        // already computes this CTA's next tile.
        named_bar_sync(1, 128);
        if (threadIdx.x == 64) {
          fence_acq_rel_sys();
          ar_signal(ar, tile);
          s_ar_ok = ar_wait(ar, tile) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (s_ar_ok && row < M) {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + n0;
#pragma unroll 4
          for (int c = 0; c < BN; c += 8)
            *reinterpret_cast<uint4*>(dst + c) = ar_load_sum8(ar, (size_t)row * N + n0 + c);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
  }
}

// Sum over ranks of 4 bf16 at element offset `off` of the slot (fp32 accumulation).
__device__ __forceinline__ uint2 ar_load_sum4(const ArArgs& ar, size_t off) {
  uint2 r;
  if (ar.mc != nullptr) {
    asm volatile("multimem.ld_reduce.weak.global.add.acc::f32.v2.bf16x2 {%0, %1}, [%2];"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(ar.mc + off)
                 : "memory");
    return r;
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k = 0; k < ar.world; ++k) {
    uint2 v;
    asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(ar.peer[k] + off)
                 : "memory");
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] += __bfloat162float(b[e]);
  }
  return make_uint2(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]));
}

// Split-K finalisation fused with the tensor-parallel all-reduce (persistent:
// the grid never exceeds what is resident, and every rank walks the items in
// the same order, so the cross-rank waits cannot deadlock).  Item = one row x
// 1024 columns: sum the split slabs, publish the bf16 partial in this rank's
// symmetric slot, signal, wait for every rank's same item, read the sum.
static __global__ void __launch_bounds__(256) splitk_finalize_ar_kernel(const float* __restrict__ ws,
                                                                 __nv_bfloat16* __restrict__ out, int M, int N,
                                                                 int64_t ldd, int splits, ArArgs ar) {
  __shared__ volatile int ok;
  const size_t slab = (size_t)M * N;
  const int chunks = (N + 1023) / 1024;
  const int items = M * chunks;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int row = item / chunks;
    const int col = (item % chunks) * 1024 + threadIdx.x * 4;
    if (col < N) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp = 0; sp < splits; ++sp) {
        const float4 p = *reinterpret_cast<const float4*>(ws + sp * slab + (size_t)row * N + col);
        v.x += p.x;
        v.y += p.y;
        v.z += p.z;
        v.w += p.w;
      }
      *reinterpret_cast<uint2*>(ar.local + (size_t)row * N + col) =
          make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_acq_rel_sys();
      ar_signal(ar, item);
      ok = ar_wait(ar, item) ? 1 : 0;
    }
    __syncthreads();
    if (ok && col < N) *reinterpret_cast<uint2*>(out + (size_t)row * ldd + col) = ar_load_sum4(ar, (size_t)row * N + col);
    __syncthreads();
  }
}

// Split-K finalisation: sum the per-split fp32 slabs in split order and write
// the real output (bf16, fp32, or SwiGLU of the interleaved gate/up columns).
template <int EPI>
__global__ void splitk_finalize_kernel(const float* __restrict__ ws, void* __restrict__ out, int M, int N,
                                       int64_t ldd, int splits) {
  const int row = blockIdx.y;
  const size_t slab = (size_t)M * N;
  if (EPI == kSwiGLU) {
    const int half = N / 2;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < half; j += gridDim.x * blockDim.x) {
      const int grp = j >> 5, off = j & 31;
      const float* pg = ws + (size_t)row * N + grp * 64 + off;
      float g = 0.f, u = 0.f;
      for (int s = 0; s < splits; ++s) {
        g += pg[s * slab];
        u += pg[s * slab + 32];
      }
      reinterpret_cast<__nv_bfloat16*>(out)[(size_t)row * ldd + j] = __float2bfloat16(silu(g) * u);
    }
  } else {
    for (int j = (blockIdx.x * blockDim.x + threadIdx.x) * 4; j < N; j += gridDim.x * blockDim.x * 4) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < splits; ++s) {
        const float4 p = *reinterpret_cast<const float4*>(ws + s * slab + (size_t)row * N + j);
        v.x += p.x;
        v.y += p.y;
        v.z += p.z;
        v.w += p.w;
      }
      if (EPI == kStoreF32) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)row * ldd + j) = v;
      } else {
        uint2 pk = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + j) = pk;
      }
    }
  }
}

}  // namespace gemm
}  // namespace lf
