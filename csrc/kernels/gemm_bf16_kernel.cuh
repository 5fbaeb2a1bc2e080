// Device code of the tcgen05 bf16 GEMM: the persistent warp-specialised
// kernel and the split-K finalize kernel (see gemm_bf16.cu for the design).
// Shared by the host launchers in gemm_bf16.cu and gemm_noalloc.cu.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_bf16.h"
#include "ll_words.cuh"

namespace lf {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;                 // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;                 // TMA warp, MMA warp, 4 epilogue warps

enum Epi : int {
  kStoreBf16 = 0,
  kStoreF32 = 1,
  kSwiGLU = 2,
  kSplitF32 = 3,
  kAllReduceBf16 = 4,
  kAllReduceLL = 5,
  kQkvRope = 6,  // QKV projection: RoPE on Q / K, K / V into the paged cache (RopeArgs)
};

// The fused all-reduce adds 4 communication warps (6..9).
constexpr int threads_for(int epi) { return epi == kAllReduceBf16 ? kThreads + 128 : kThreads; }

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Arrival / completion signals of the fused all-reduce (see ArArgs).  The
// caller has ordered its data stores before the signal (barrier + fence).
__device__ __forceinline__ void ar_signal_one(const ArArgs& ar, int r, int idx) {
  asm volatile("red.release.sys.global.add.s32 [%0], 1;" ::"l"(ar.cnt_peer[r] + idx) : "memory");
}
__device__ __forceinline__ void ar_signal_all(const ArArgs& ar, int idx) {
  if (ar.cnt_mc != nullptr) {
    asm volatile("multimem.red.release.sys.global.add.s32 [%0], 1;" ::"l"(ar.cnt_mc + idx) : "memory");
  } else {
    for (int r = 0; r < ar.world; ++r) ar_signal_one(ar, r, idx);
  }
}

// Waits (bounded) until counter `idx` reaches `target`, then re-arms it.
// Returns false after recording kErrPeerTimeout.
__device__ __forceinline__ bool ar_wait(const ArArgs& ar, int idx, int target) {
  int* c = ar.cnt_local + idx;
  if (ld_acquire_sys(c) < target) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys(c) < target) {
      if ((++spins & 63u) == 0) {
        if (error_pending()) return false;
        if (globaltimer_ns() - t0 > wait_limit_ns()) {
          set_error(kErrPeerTimeout, (unsigned long long)idx);
          return false;
        }
      }
    }
  }
  // Every signal of this use has arrived, and none of the next use of the
  // counter can come before this rank starts that use: a plain re-arm is safe.
  atomicSub(c, target);
  return true;
}

// Owner rank of an output tile: dealt round-robin (all-reduce), or by rows
// (reduce-scatter mode).
__device__ __forceinline__ int ar_owner(const ArArgs& ar, int tile, int num_m, int bm) {
  return ar.rs_rows > 0 ? ((tile % num_m) * bm) / ar.rs_rows : tile % ar.world;
}

// Sum over ranks of the 8 bf16 partials at element offset `off` (fp32 accumulation).
__device__ __forceinline__ uint4 ar_reduce8(const ArArgs& ar, size_t off) {
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

// Writes 8 reduced bf16 into every rank's result region at offset `off`.
__device__ __forceinline__ void ar_store8(const ArArgs& ar, size_t off, uint4 v) {
  if (ar.out_mc != nullptr) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(ar.out_mc + off),
                 "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
    return;
  }
  for (int k = 0; k < ar.world; ++k) *reinterpret_cast<uint4*>(ar.out_peer[k] + off) = v;
}

// MB: 128-row M-blocks per tile (2: a 256-row tile whose two MMAs share each
// staged B slab, so a skinny GEMM streams its weights once instead of once
// per M-block).
template <int BN, int STAGES, int MB = 1>
struct Smem {
  static constexpr int kABytes = MB * BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTotal = STAGES * kStageBytes + 1024 /*align slack*/ + 256 /*barriers*/;
};

// Accumulators in flight per CTA: two (epilogue of one tile overlaps the
// MMAs of the next) when they fit the 512 TMEM columns, else one.
template <int BN, int MB>
constexpr int tmem_accs() {
  return 2 * MB * BN <= 512 ? 2 : 1;
}

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

// Rotation of one (x1, x2) split-half pair by the angle whose (cos, sin) is cs.
__device__ __forceinline__ float2 rope_pair(float x1, float x2, float2 cs) {
  return make_float2(x1 * cs.x - x2 * cs.y, x2 * cs.x + x1 * cs.y);
}

// kQkvRope epilogue of the persistent kernel: the thread owns one row (TMEM
// lane) of a tile whose BN columns are BN / 128 whole heads.  tcgen05.ld is
// warp-collective, so every lane loads and only live rows store.
template <int BN>
__device__ __forceinline__ void qkv_rope_row(const RopeArgs& rp, uint32_t taddr, int row, int M, int n0,
                                             __nv_bfloat16* __restrict__ out, int ldd) {
  static_assert(BN % 128 == 0, "whole heads per tile");
  const bool live = row < M;
  const int pos = live ? rp.positions[row] : 0;
  const int slot = live ? rp.slots[row] : -1;
  const bool pos_ok = pos >= 0 && pos < rp.max_pos;
  if (live && !pos_ok) set_error(kErrBadIndex, (unsigned long long)row);
  const bool slot_ok = slot >= 0 && (int64_t)slot < rp.num_slots;
  const int pg = slot_ok ? slot / rp.page : 0, off = slot_ok ? slot % rp.page : 0;
#pragma unroll 1
  for (int j = 0; j < BN / 128; ++j) {
    const int hd = n0 / 128 + j;
    const bool is_q = hd < rp.Hq;
    const bool is_v = hd >= rp.Hq + rp.Hkv;
    __nv_bfloat16* dst;
    if (is_q) {
      dst = out + (size_t)row * ldd + (size_t)hd * 128;
    } else {
      const int kh = is_v ? hd - rp.Hq - rp.Hkv : hd - rp.Hq;
      dst = (is_v ? rp.vcache : rp.kcache) + (((size_t)pg * rp.Hkv + kh) * rp.page + off) * 128;
    }
    const bool write = live && (is_q || slot_ok);
#pragma unroll 1
    for (int c = 0; c < 64; c += 32) {
      uint32_t x1[32], x2[32];
      tmem_ld_32x32b_x32(taddr + j * 128 + c, x1);
      tmem_ld_32x32b_x32(taddr + j * 128 + 64 + c, x2);
      tmem_wait_ld();
      if (!write) continue;
      uint32_t p1[16], p2[16];
      if (!is_v) {
        const float4* cs4 = reinterpret_cast<const float4*>(rp.cos_sin + (size_t)(pos_ok ? pos : 0) * 64 + c);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          // (cos, sin) of pairs c + 2e and c + 2e + 1
          const float4 cs = pos_ok ? cs4[e] : make_float4(1.f, 0.f, 1.f, 0.f);
          const float2 r0 = rope_pair(__uint_as_float(x1[2 * e]), __uint_as_float(x2[2 * e]), make_float2(cs.x, cs.y));
          const float2 r1 =
              rope_pair(__uint_as_float(x1[2 * e + 1]), __uint_as_float(x2[2 * e + 1]), make_float2(cs.z, cs.w));
          p1[e] = pack_bf16x2(r0.x, r1.x);
          p2[e] = pack_bf16x2(r0.y, r1.y);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          p1[e] = pack_bf16x2(__uint_as_float(x1[2 * e]), __uint_as_float(x1[2 * e + 1]));
          p2[e] = pack_bf16x2(__uint_as_float(x2[2 * e]), __uint_as_float(x2[2 * e + 1]));
        }
      }
      uint4* d1 = reinterpret_cast<uint4*>(dst + c);
      uint4* d2 = reinterpret_cast<uint4*>(dst + 64 + c);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        d1[e] = make_uint4(p1[4 * e], p1[4 * e + 1], p1[4 * e + 2], p1[4 * e + 3]);
        d2[e] = make_uint4(p2[4 * e], p2[4 * e + 1], p2[4 * e + 2], p2[4 * e + 3]);
      }
    }
  }
}

template <int BN, int STAGES, int EPI, int MB = 1>
__global__ void __launch_bounds__(threads_for(EPI), 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b, void* __restrict__ out, int M,
                     int N, int K, int ldd, int splits, int kb_per_split, ArArgs ar,
                     const int* __restrict__ groups, int num_groups, const RopeArgs rope) {
  // Grouped mode (groups != nullptr, mixture-of-experts): A's rows are split
  // into num_groups segments, groups[g]..groups[g+1] (each a multiple of BM,
  // read from device memory), and segment g multiplies B rows [g*N, (g+1)*N).
  // M is then an upper bound on groups[num_groups]; blocks past it are skipped.
  static_assert(MB == 1 || (EPI != kSplitF32 && EPI != kAllReduceBf16), "256-row tiles: plain epilogues only");
  pdl_trigger();
  using S = Smem<BN, STAGES, MB>;
  constexpr int kAccs = tmem_accs<BN, MB>();
  constexpr int TM = MB * BM;                 // rows per tile
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + TM - 1) / TM;
  const int num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles * splits;
  const int num_kb = (K + BK - 1) / BK;
  constexpr uint32_t kCols = MB == 1 ? tmem_cols<BN>() : 512;

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
  pdl_wait();  // the set-up above touches no global memory
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
        const int m0 = (tile % num_m) * TM;
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
#pragma unroll
          for (int j = 0; j < MB; ++j) tma_load_2d(sa + j * BM * BK * 2, &tmap_a, &full_bar[stage], kb * BK, m0 + j * BM);
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
        const int acc = kAccs == 2 ? (local & 1) : 0;
        const uint32_t acc_phase = kAccs == 2 ? ((local >> 1) & 1) : (local & 1);
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * MB * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
            for (int j = 0; j < MB; ++j)
              umma_f16_ss(d_tmem + j * BN, sw128_kmajor_desc(sa + j * BM * BK * 2 + kk * 32),
                          sw128_kmajor_desc(sb + kk * 32), idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
    }
  } else if (warp < 6) {
    // Epilogue warps 2..5 -> TMEM lane quadrant (warp % 4).
    const int quad = warp & 3;
    int local = 0;
    for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x, ++local) {
      const int tile = unit % num_tiles;
      if (groups != nullptr && group_of(groups, num_groups, (tile % num_m) * BM) < 0) {
        --local;
        continue;
      }
      const int acc = kAccs == 2 ? (local & 1) : 0;
      const uint32_t acc_phase = kAccs == 2 ? ((local >> 1) & 1) : (local & 1);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, 4)) break;
      tc_fence_after();
      const int n0 = (tile / num_m) * BN;
#pragma unroll 1
      for (int mb = 0; mb < MB; ++mb) {
      const int m0 = (tile % num_m) * TM + mb * BM;
      const int row = m0 + quad * 32 + lane;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * MB * BN + mb * BN;
      if constexpr (EPI == kQkvRope) {
        qkv_rope_row<BN>(rope, taddr, row, M, n0, reinterpret_cast<__nv_bfloat16*>(out), ldd);
      } else if constexpr (EPI == kSwiGLU) {
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
              // kAllReduceBf16 publishes the partial tile in this rank's
              // symmetric partial region (row stride N).
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
      }  // M-blocks of the tile
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);  // the MMA warp may start the next tile now
      if constexpr (EPI == kAllReduceBf16) {
        // The partial tile is published: signal the tile's owner rank (tiles
        // are dealt round-robin over the ranks) and go on with the next tile.
        named_bar_sync(1, 128);
        if (threadIdx.x == 64) {
          fence_acq_rel_sys();
          ar_signal_one(ar, ar_owner(ar, tile, num_m, BM), tile);
          if (ar.trace != nullptr) ar.trace[4 * tile] = globaltimer_ns();
        }
      }
    }
  } else if constexpr (EPI == kAllReduceBf16) {
    // Communication warps 6..9: for every tile this rank owns, wait for all
    // ranks' partials, read their sum through the switch and write it into
    // every rank's result region, then signal completion to every rank.  They
    // trail the epilogue without ever blocking it or the MMA warp.
    const int t = threadIdx.x - 192;
    for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x) {
      const int tile = unit % num_tiles;
      if (ar_owner(ar, tile, num_m, BM) != ar.rank) continue;
      if (t == 0) {
        s_ar_ok = ar_wait(ar, tile, ar.world) ? 1 : 0;
        if (ar.trace != nullptr) ar.trace[4 * tile + 1] = globaltimer_ns();
      }
      named_bar_sync(2, 128);
      if (s_ar_ok) {
        // Coalesced over the tile (consecutive threads, consecutive 16-byte
        // vectors of a row); up to 16 switch reductions in flight per
        // thread before their results are stored.
        const int m0 = (tile % num_m) * BM;
        const int n0 = (tile / num_m) * BN;
        constexpr int kVecs = BN / 8;
        constexpr int kIters = BM * kVecs / 128;
        constexpr int kBatch = kIters < 16 ? kIters : 16;
#pragma unroll 1
        for (int it = 0; it < kIters; it += kBatch) {
          uint4 v[kBatch];
          size_t off[kBatch];
#pragma unroll
          for (int j = 0; j < kBatch; ++j) {
            const int i = (it + j) * 128 + t;
            const int r = m0 + i / kVecs;
            off[j] = r < M ? (size_t)r * N + n0 + (i % kVecs) * 8 : ~size_t(0);
            if (r < M) v[j] = ar_reduce8(ar, off[j]);
          }
#pragma unroll
          for (int j = 0; j < kBatch; ++j) {
            if (off[j] == ~size_t(0)) continue;
            if (ar.rs_rows > 0) {
              // reduce-scatter: the owner keeps its rows
              *reinterpret_cast<uint4*>(ar.rs_out + off[j] - (size_t)ar.rank * ar.rs_rows * N) = v[j];
            } else {
              ar_store8(ar, off[j], v[j]);
            }
          }
        }
      }
      named_bar_sync(2, 128);
      if (t == 0) {
        fence_acq_rel_sys();
        ar_signal_all(ar, ar.cnt_capacity + tile);
        if (ar.trace != nullptr) {
          ar.trace[4 * tile + 2] = globaltimer_ns();
          ar.trace[4 * tile + 3] = blockIdx.x + 1;
        }
      }
    }
    // The kernel ends only when the owners of this CTA's tiles have written
    // their sums everywhere, so the next kernel on this stream sees them.
    if (t == 0) {
      for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x)
        if (!ar_wait(ar, ar.cnt_capacity + unit % num_tiles, 1)) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
  }
}

// ---------------------------------------------------------------------------
// Cluster split-K for skinny (decode) GEMMs.  One thread-block cluster of c
// CTAs per output tile, CTA r of the cluster computes K slice r into its own
// TMEM accumulator; the partial tiles are then summed through distributed
// shared memory (each CTA owns 1/c of the tile's rows and reads that band of
// every peer's partial, in cluster-rank order, so the result is
// deterministic) and written once, in the final format.  No fp32 workspace
// round trip through HBM and no second kernel.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_shared_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int BN>
struct ClusterRed {
  static constexpr int kStride = BN + 4;  // fp32 row stride of the partial tile (bank spread)
  static constexpr int kBytes = BM * kStride * 4;
};

// Sum of the cluster's partials for 4 consecutive columns of one row.
template <int BN>
__device__ __forceinline__ float4 cluster_sum4(uint32_t red_base, int c, int rl, int col) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const uint32_t off = red_base + (uint32_t)(rl * ClusterRed<BN>::kStride + col) * 4;
  for (int q = 0; q < c; ++q) {
    const float4 a = ld_shared_cluster_f4(mapa_shared(off, q));
    acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
  }
  return acc;
}

// kQkvRope epilogue of the cluster kernel: thread t of the 128 epilogue
// threads takes (row, head of the tile, 4 consecutive split-half pairs) items
// of its CTA's band of rows [r0, r1), sums the cluster's partials for the 4
// first-half and the 4 matching second-half columns, rotates (Q, K) or copies
// (V) them and stores Q to `out`, K / V into the paged cache.
template <int BN>
__device__ __forceinline__ void qkv_rope_cluster(const RopeArgs& rp, uint32_t red_base, int c, int r0, int r1,
                                                 int mrow0, int n0, int M, __nv_bfloat16* __restrict__ out, int ldd,
                                                 int t) {
  static_assert(BN % 128 == 0, "whole heads per tile");
  constexpr int kHeads = BN / 128;
  constexpr int kPerRow = kHeads * 16;
  for (int i = t; i < (r1 - r0) * kPerRow; i += 128) {
    const int rl = r0 + i / kPerRow;
    const int j = (i / 16) % kHeads;
    const int q = (i % 16) * 4;  // first of the 4 pairs
    const int grow = mrow0 + rl;
    if (grow >= M) continue;
    const int hd = n0 / 128 + j;
    const bool is_q = hd < rp.Hq;
    const bool is_v = hd >= rp.Hq + rp.Hkv;
    const int pos = rp.positions[grow];
    const int slot = rp.slots[grow];
    const bool pos_ok = pos >= 0 && pos < rp.max_pos;
    if (!pos_ok && q == 0 && j == 0) set_error(kErrBadIndex, (unsigned long long)grow);
    const bool slot_ok = slot >= 0 && (int64_t)slot < rp.num_slots;
    if (!is_q && !slot_ok) continue;
    const float4 a = cluster_sum4<BN>(red_base, c, rl, j * 128 + q);
    const float4 b = cluster_sum4<BN>(red_base, c, rl, j * 128 + 64 + q);
    float o1[4] = {a.x, a.y, a.z, a.w}, o2[4] = {b.x, b.y, b.z, b.w};
    if (!is_v) {
      const float4* cs4 = reinterpret_cast<const float4*>(rp.cos_sin + (size_t)(pos_ok ? pos : 0) * 64 + q);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float4 cs = pos_ok ? cs4[e] : make_float4(1.f, 0.f, 1.f, 0.f);
        const float2 r0v = rope_pair(o1[2 * e], o2[2 * e], make_float2(cs.x, cs.y));
        const float2 r1v = rope_pair(o1[2 * e + 1], o2[2 * e + 1], make_float2(cs.z, cs.w));
        o1[2 * e] = r0v.x;
        o2[2 * e] = r0v.y;
        o1[2 * e + 1] = r1v.x;
        o2[2 * e + 1] = r1v.y;
      }
    }
    __nv_bfloat16* dst;
    if (is_q) {
      dst = out + (size_t)grow * ldd + (size_t)hd * 128;
    } else {
      const int kh = is_v ? hd - rp.Hq - rp.Hkv : hd - rp.Hq;
      const int pg = slot / rp.page, off = slot % rp.page;
      dst = (is_v ? rp.vcache : rp.kcache) + (((size_t)pg * rp.Hkv + kh) * rp.page + off) * 128;
    }
    *reinterpret_cast<uint2*>(dst + q) = make_uint2(pack_bf16x2(o1[0], o1[1]), pack_bf16x2(o1[2], o1[3]));
    *reinterpret_cast<uint2*>(dst + 64 + q) = make_uint2(pack_bf16x2(o2[0], o2[1]), pack_bf16x2(o2[2], o2[3]));
  }
}

// Epilogue of the fused decode all-reduce (kAllReduceLL), run by the 128
// epilogue threads (t) of a CTA on its band of rows [r0, r1) of the tile.
// Output pairs (two bf16 of one row) are numbered p = (row * N + col) / 2 and
// dealt to the ranks in contiguous chunks, exactly as the standalone kernel
// does, so the two share inboxes and epochs:
//   1. every pair owned by another rank: this rank's bf16 partial -> the
//      owner's reduce-scatter inbox (one 8-byte store with the epoch);
//   2. every pair this rank owns: its own partial (rounded to bf16 like the
//      others) plus the other ranks' inbox words, stored to `out` and to every
//      rank's all-gather inbox (one multicast store, or one per peer);
//   3. every pair owned by another rank: the owner's all-gather word -> `out`.
// Step 2 waits only for step 1 of the other ranks and step 3 only for step 2,
// and no rank waits before finishing its step 1, so the waits form no cycle
// across ranks; every wait is bounded.
template <int BN>
__device__ __forceinline__ void ll_epilogue(const ar::LLArgs& ll, uint32_t ep, uint32_t red_base, int c, int r0,
                                            int r1, int mrow0, int n0, int M, int N, int ldd,
                                            __nv_bfloat16* __restrict__ out, int t) {
  constexpr int kQuads = BN / 4;
  const int64_t P = (int64_t)M * N / 2;
  const int64_t chunk = (P + ll.world - 1) / ll.world;
  const int64_t p_lo = ll.rank * chunk;
  const int64_t p_hi = p_lo + chunk < P ? p_lo + chunk : P;
  const int n_items = (r1 - r0) * kQuads;
  // 1. partials of the pairs other ranks own
  for (int i = t; i < n_items; i += 128) {
    const int rl = r0 + i / kQuads;
    const int col = (i % kQuads) * 4;
    const int grow = mrow0 + rl;
    if (grow >= M) continue;
    const int64_t p = ((int64_t)grow * N + n0 + col) >> 1;
    if (p >= p_lo && p + 1 < p_hi) continue;  // both pairs are this rank's
    const float4 acc = cluster_sum4<BN>(red_base, c, rl, col);
    const uint32_t w[2] = {ar::pack2(acc.x, acc.y), ar::pack2(acc.z, acc.w)};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int64_t pp = p + e;
      const int owner = (int)(pp / chunk);
      if (owner != ll.rank) ar::st_word(ll.rs[owner] + (int64_t)ll.rank * chunk + (pp - owner * chunk), w[e], ep);
    }
  }
  // 2. the pairs this rank owns
  bool ok = true;
  for (int i = t; i < n_items && ok; i += 128) {
    const int rl = r0 + i / kQuads;
    const int col = (i % kQuads) * 4;
    const int grow = mrow0 + rl;
    if (grow >= M) continue;
    const int64_t p = ((int64_t)grow * N + n0 + col) >> 1;
    if (p + 1 < p_lo || p >= p_hi) continue;  // neither pair is this rank's
    const float4 acc = cluster_sum4<BN>(red_base, c, rl, col);
    const float2 own[2] = {make_float2(acc.x, acc.y), make_float2(acc.z, acc.w)};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int64_t pp = p + e;
      if (pp < p_lo || pp >= p_hi || !ok) continue;
      float2 sum = ar::unpack2(ar::pack2(own[e].x, own[e].y));  // the same bf16 rounding as every rank's partial
      for (int src = 0; src < ll.world; ++src) {
        if (src == ll.rank) continue;
        uint32_t d;
        if (!ar::poll_word(ll.rs[ll.rank] + (int64_t)src * chunk + (pp - p_lo), ep, &d)) {
          ok = false;
          break;
        }
        const float2 v = ar::unpack2(d);
        sum.x += v.x;
        sum.y += v.y;
      }
      if (!ok) break;
      const uint32_t r = ar::pack2(sum.x, sum.y);
      *reinterpret_cast<uint32_t*>(out + (size_t)grow * ldd + n0 + col + 2 * e) = r;
      if (ll.ag_mc != nullptr) {
        ar::st_word_mc(ll.ag_mc + pp, r, ep);
      } else {
        for (int k = 0; k < ll.world; ++k)
          if (k != ll.rank) ar::st_word(ll.ag[k] + pp, r, ep);
      }
    }
  }
  // 3. the pairs other ranks own
  for (int i = t; i < n_items && ok; i += 128) {
    const int rl = r0 + i / kQuads;
    const int col = (i % kQuads) * 4;
    const int grow = mrow0 + rl;
    if (grow >= M) continue;
    const int64_t p = ((int64_t)grow * N + n0 + col) >> 1;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int64_t pp = p + e;
      if (pp >= p_lo && pp < p_hi) continue;
      uint32_t d;
      if (!ar::poll_word(ll.ag[ll.rank] + pp, ep, &d)) {
        ok = false;
        break;
      }
      *reinterpret_cast<uint32_t*>(out + (size_t)grow * ldd + n0 + col + 2 * e) = d;
    }
  }
}


// OUT: kStoreBf16, kStoreF32, kSwiGLU (interleaved gate/up groups of 32), or
// kAllReduceLL: bf16 out = sum over the tensor-parallel ranks, the epilogue
// running the low-latency all-reduce protocol itself (`ll`, see
// allreduce_ll.cu) on the cluster-reduced values, so the row-parallel decode
// projection and its all-reduce are one kernel.
// MB: 128-row M-blocks per tile.  With MB = 2 (decode batches of 129..256
// rows) the two MMAs of a k-slab share the staged weight slab, so the weights
// cross into shared memory once instead of once per M-block; the two partial
// M-blocks are then reduced one after the other through the same staging
// buffer (it holds one 128-row partial).
template <int BN, int STAGES, int OUT, int MB = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_cluster_splitk_kernel(const __grid_constant__ CUtensorMap tmap_a,
                               const __grid_constant__ CUtensorMap tmap_b, void* __restrict__ out, int M, int N,
                               int K, int ldd, int kb_per_split, const ar::LLArgs ll, const RopeArgs rope) {
  using S = Smem<BN, STAGES, MB>;
  static_assert(ClusterRed<BN>::kBytes <= STAGES * S::kStageBytes, "partial tile must fit the pipeline buffers");
  static_assert(MB * BN <= 512, "accumulators must fit TMEM");
  static_assert(OUT != kAllReduceLL || MB == 1, "fused all-reduce: 128-row tiles");
  pdl_trigger();
  constexpr int TM = MB * BM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull_bar + 1);
  float* red = reinterpret_cast<float*>(smem);  // the partial tile, once the pipeline has drained

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c = (int)cluster_nctarank();
  const int r = (int)cluster_ctarank();
  const int num_m = (M + TM - 1) / TM;
  const int tile = blockIdx.x / c;
  const int m0 = (tile % num_m) * TM;
  const int n0 = (tile / num_m) * BN;
  const int num_kb = (K + BK - 1) / BK;
  const int kb0 = r * kb_per_split;
  const int kb1 = min(num_kb, kb0 + kb_per_split);
  constexpr uint32_t kCols = MB * BN < 32 ? 32 : MB * BN;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    for (int st = 0; st < STAGES; ++st) {
      mbar_init(&full_bar[st], 1);
      mbar_init(&empty_bar[st], 1);
    }
    mbar_init(tfull_bar, 1);
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
  // The weight slabs do not depend on the previous kernel: the first stages'
  // B loads go out before the dependency wait (under programmatic dependent
  // launch they overlap the previous kernel's tail); their A loads follow it.
  const int pre = (warp == 0 && lane == 0) ? min(STAGES, kb1 - kb0) : 0;
  const uint64_t pol_b = l2_policy_evict_first();
  for (int i = 0; i < pre; ++i) {
    mbar_arrive_expect_tx(&full_bar[i], S::kStageBytes);
    tma_load_2d_hint(smem + i * S::kStageBytes + S::kABytes, &tmap_b, &full_bar[i], (kb0 + i) * BK, n0, pol_b);
  }
  pdl_wait();  // everything above touches no memory the previous kernel writes
  // fused all-reduce: this operation's epoch (advanced by the grid's last CTA)
  uint32_t ep = 0;
  if constexpr (OUT == kAllReduceLL) ep = (uint32_t)(*reinterpret_cast<volatile int*>(ll.state)) + 1u;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        uint8_t* sa = smem + stage * S::kStageBytes;
        uint8_t* sb = sa + S::kABytes;
        if (kb - kb0 >= pre) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, 11)) break;
          mbar_arrive_expect_tx(&full_bar[stage], S::kStageBytes);
          tma_load_2d_hint(sb, &tmap_b, &full_bar[stage], kb * BK, n0, pol_b);
        }
#pragma unroll
        for (int j = 0; j < MB; ++j) tma_load_2d(sa + j * BM * BK * 2, &tmap_a, &full_bar[stage], kb * BK, m0 + j * BM);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, 12)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
        const uint32_t sb = sa + S::kABytes;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
          for (int j = 0; j < MB; ++j)
            umma_f16_ss(tmem_base + j * BN, sw128_kmajor_desc(sa + j * BM * BK * 2 + kk * 32),
                        sw128_kmajor_desc(sb + kk * 32), idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      // commit also when the slice was empty or a wait failed, so the
      // epilogue never waits for nothing (it then writes zeros)
      if (ok) umma_commit(tfull_bar);
      else mbar_arrive(tfull_bar);
    }
  }
  const int quad = warp & 3;
  const bool have = kb1 > kb0;
  bool acc_ok = false;
  if (warp >= 2) {
    acc_ok = mbar_wait(tfull_bar, 0, 13);
    if (acc_ok) tc_fence_after();
  }
  // Every CTA runs the same 2 * MB cluster barriers below (uniform control flow).
#pragma unroll 1
  for (int mb = 0; mb < MB; ++mb) {
    if (warp >= 2 && acc_ok) {
      // TMEM -> this CTA's fp32 partial of M-block mb in shared memory (row = TMEM lane)
      const int row = quad * 32 + lane;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + mb * BN;
      float* dst = red + row * ClusterRed<BN>::kStride;
#pragma unroll 1
      for (int col = 0; col < BN; col += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + col, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 f = have ? make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                        __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(dst + col + 4 * j) = f;
        }
      }
    }
    // every CTA's partial of this M-block is in its shared memory
    cluster_sync_all();
    if (warp >= 2) {
      const int t = threadIdx.x - 64;
      const int rows_per = (BM + c - 1) / c;
      const int r0 = r * rows_per;
      const int r1 = min(BM, r0 + rows_per);
      const int mrow0 = m0 + mb * BM;
      const uint32_t red_base = smem_u32(red);
      if constexpr (OUT == kSwiGLU) {
        // thread -> (row, 4 consecutive output features): gate cols g*64 + j,
        // up cols g*64 + 32 + j of the tile
        constexpr int kQuads = BN / 2 / 4;
        // unrolled: several iterations' remote loads in flight per thread
#pragma unroll 4
        for (int i = t; i < (r1 - r0) * kQuads; i += 128) {
          const int rl = r0 + i / kQuads;
          const int j = (i % kQuads) * 4;            // output feature within the tile
          const int gcol = (j / 32) * 64 + (j % 32);
          float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
          const uint32_t off_g = red_base + (uint32_t)(rl * ClusterRed<BN>::kStride + gcol) * 4;
          for (int q = 0; q < c; ++q) {
            const float4 a = ld_shared_cluster_f4(mapa_shared(off_g, q));
            const float4 b = ld_shared_cluster_f4(mapa_shared(off_g + 32 * 4, q));
            g.x += a.x; g.y += a.y; g.z += a.z; g.w += a.w;
            u.x += b.x; u.y += b.y; u.z += b.z; u.w += b.w;
          }
          const int grow = mrow0 + rl;
          if (grow < M) {
            __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)grow * ldd + n0 / 2 + j;
            *reinterpret_cast<uint2*>(d) =
                make_uint2(pack_bf16x2(silu(g.x) * u.x, silu(g.y) * u.y), pack_bf16x2(silu(g.z) * u.z, silu(g.w) * u.w));
          }
        }
      } else if constexpr (OUT == kAllReduceLL) {
        ll_epilogue<BN>(ll, ep, red_base, c, r0, r1, mrow0, n0, M, N, ldd, reinterpret_cast<__nv_bfloat16*>(out), t);
      } else if constexpr (OUT == kQkvRope) {
        qkv_rope_cluster<BN>(rope, red_base, c, r0, r1, mrow0, n0, M, reinterpret_cast<__nv_bfloat16*>(out), ldd, t);
      } else {
        constexpr int kQuads = BN / 4;
        // unrolled: several iterations' remote loads in flight per thread
#pragma unroll 4
        for (int i = t; i < (r1 - r0) * kQuads; i += 128) {
          const int rl = r0 + i / kQuads;
          const int col = (i % kQuads) * 4;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          const uint32_t off = red_base + (uint32_t)(rl * ClusterRed<BN>::kStride + col) * 4;
          for (int q = 0; q < c; ++q) {
            const float4 a = ld_shared_cluster_f4(mapa_shared(off, q));
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
          }
          const int grow = mrow0 + rl;
          if (grow < M) {
            if constexpr (OUT == kStoreF32) {
              *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)grow * ldd + n0 + col) = acc;
            } else {
              *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)grow * ldd + n0 + col) =
                  make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
            }
          }
        }
      }
    }
    // no CTA overwrites its staging buffer (next M-block) or leaves (and
    // releases its shared memory) while a peer still reads it
    if (mb + 1 == MB) tc_fence_before();
    cluster_sync_all();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
  }
  if constexpr (OUT == kAllReduceLL) {
    // advance the epoch once every CTA has read it (all have passed the
    // cluster barrier above, which follows their read)
    if (threadIdx.x == 0 && atomicAdd(ll.state + 1, 1) == (int)gridDim.x - 1) {
      ll.state[1] = 0;
      *reinterpret_cast<volatile int*>(ll.state) = (int)ep;
    }
  }
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Counters of the finalize kernel, at the top of the arrival half (the tile
// path keeps below them): two cross-rank barriers, and the arrival count and
// generation of this rank's grid barrier.
constexpr int kFinReserved = 4;

// Barrier over every CTA of this grid and every rank: each CTA makes its
// stores visible system-wide and arrives on a local counter; the last CTA to
// arrive signals every rank on counter `xidx`, waits for all of them, and
// releases this rank's CTAs by bumping the generation.  One cross-rank round
// trip per rank, whatever the grid size.  Needs every CTA resident.
__device__ __forceinline__ bool grid_rank_barrier(const ArArgs& ar, int xidx) {
  __shared__ volatile int s_ok;
  int* arrive = ar.cnt_local + ar.cnt_capacity - 2;
  int* gen = ar.cnt_local + ar.cnt_capacity - 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    bool ok = true;
    fence_acq_rel_sys();
    const int g = ld_acquire_gpu(gen);
    if (atom_add_acq_rel_gpu(arrive, 1) == (int)gridDim.x - 1) {
      atomicExch(arrive, 0);
      ar_signal_all(ar, xidx);
      ok = ar_wait(ar, xidx, ar.world);
      st_release_gpu(gen, g + 1);
    } else if (ld_acquire_gpu(gen) == g) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu(gen) == g) {
        if ((++spins & 63u) == 0 && (error_pending() || globaltimer_ns() - t0 > wait_limit_ns())) {
          if (!error_pending()) set_error(kErrPeerTimeout, (unsigned long long)xidx);
          ok = false;
          break;
        }
      }
    }
    s_ok = ok ? 1 : 0;
  }
  __syncthreads();
  return s_ok != 0;
}

// Split-K finalisation fused with the tensor-parallel all-reduce, over the
// flattened [M, N] output in 8-element vectors (persistent grid, every CTA
// resident, same grid on every rank):
//   1. sum the split slabs, publish the bf16 partials;   barrier
//   2. reduce this rank's 1/world of the output through the switch and write
//      it into every rank's result region (8 reductions in flight a thread);
//                                                         barrier
// Two cross-rank round trips per operation.
static __global__ void __launch_bounds__(256, 2) splitk_finalize_ar_kernel(const float* __restrict__ ws, int M, int N,
                                                                 int splits, ArArgs ar) {
  const size_t slab = (size_t)M * N;
  const int64_t nvec = (int64_t)slab / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t v = first; v < nvec; v += stride) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < splits; ++sp) {
      const float4* p = reinterpret_cast<const float4*>(ws + sp * slab + v * 8);
      const float4 x = p[0], y = p[1];
      a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
      a[4] += y.x; a[5] += y.y; a[6] += y.z; a[7] += y.w;
    }
    *reinterpret_cast<uint4*>(ar.local + v * 8) =
        make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
  }
  if (!grid_rank_barrier(ar, ar.cnt_capacity - kFinReserved)) return;
  const int64_t v0 = nvec * ar.rank / ar.world, v1 = nvec * (ar.rank + 1) / ar.world;
  constexpr int kBatch = 8;
  for (int64_t base = v0 + first; base < v1; base += kBatch * stride) {
    uint4 r[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (base + j * stride < v1) r[j] = ar_reduce8(ar, (size_t)(base + j * stride) * 8);
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (base + j * stride < v1) ar_store8(ar, (size_t)(base + j * stride) * 8, r[j]);
  }
  grid_rank_barrier(ar, ar.cnt_capacity - kFinReserved + 1);
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
