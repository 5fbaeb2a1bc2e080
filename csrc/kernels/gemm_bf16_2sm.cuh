// Persistent bf16 GEMM on CTA pairs: tcgen05.mma with cta_group::2.
//
//   D[M, N] = A[M, K] . B[N, K]^T
//
// Why a pair: a single-CTA M=128 x N=256 MMA reads a 4 KB A slab and an 8 KB
// B slab from shared memory per 1 MFLOP, while TMA writes the same 12 KB into
// it, so shared memory (not the tensor core) is the limit of the 1-CTA kernel
// on large prefill GEMMs.  With cta_group::2 one MMA computes a 256 x 256 tile
// on two SMs: each CTA stages its own 128 rows of A and half (128 rows) of B,
// and the tensor cores of the pair read the other half of B from the peer.
// Shared-memory traffic per FLOP drops by a third and every weight slab is
// fetched from L2 once per 256 output rows.
//
// Roles (192 threads per CTA, one CTA pair per cluster, persistent):
//   warp 0      TMA producer, in both CTAs: this CTA's A rows and B half of
//               each k-slab.  The bytes of both CTAs complete on the leader's
//               `full` barrier (the .cta_group::2 form of the TMA load lets a
//               CTA signal its peer's barrier); only the leader posts the
//               expected byte count.
//   warp 1      allocates 512 TMEM columns in both CTAs (the pair allocation
//               is collective: same warp, same smem slot in each CTA); in the
//               leader, lane 0 issues the MMAs and commits, multicast to both
//               CTAs' barriers, to free the k-slab and to hand an accumulator
//               to the epilogues.
//   warps 2..5  epilogue, in both CTAs: each reads its 128 rows x 256 columns
//               from its own TMEM, stores, and one lane per warp arrives on
//               the leader's `tempty` barrier (8 arrivals per accumulator).
// Two accumulators (2 x 256 columns) let the epilogue of one tile overlap the
// MMAs of the next.  Every wait is bounded; every thread reaches the final
// cluster barrier, so a failed wait never leaves a peer waiting there.
//
// Reference: the reference plans its projections as external AOT modules or a
// cuBLASLt call (internal/cuda/gemm.c:108-207); this kernel has no counterpart.
//
// Included by gemm_bf16.cu (it uses that file's tensor-map cache and SM count).
#pragma once
#include <cuda.h>

#include <cstdlib>

#include "common.cuh"
#include "gemm_bf16.h"
#include "gemm_bf16_kernel.cuh"

namespace lf {
namespace gemm {
namespace pair {

constexpr int kTileM = 256;            // rows per pair tile (128 per CTA)
constexpr int kTileN = 256;            // widest pair tile (B: 128 rows per CTA); TMEM columns per accumulator
constexpr int kBoxRowsNarrow = 32;     // B rows per TMA box with 192 / 256-wide tiles (bn / 64 boxes per stage)

// Column tiling of N: `wide` tiles of base + 64 columns, then base-wide
// tiles.  Uniform 256-wide tiles for most shapes; a GEMM with one M-tile
// whose 256-wide tiles would leave pairs idle in the last round is cut into
// k tiles per pair of near-equal width (multiples of 64), so every pair gets
// the same number of tiles.
struct ColPlan {
  int tiles_n;
  int wide;
  int base;
  int box_rows;   // B rows per TMA box: 128 (one box per stage) for uniform tiles, 32 otherwise
};

__host__ __device__ __forceinline__ void tile_cols(const ColPlan& cp, int tn, int& n0, int& bn) {
  if (tn < cp.wide) {
    bn = cp.base + 64;
    n0 = tn * bn;
  } else {
    bn = cp.base;
    n0 = cp.wide * (cp.base + 64) + (tn - cp.wide) * cp.base;
  }
}
constexpr int kStageBytes = BM * BK * 2 + (kTileN / 2) * BK * 2;  // 32 KB per CTA
constexpr int kStages = 6;
constexpr int kSmem = kStages * kStageBytes + 1024 + 256;

__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// TMA load into this CTA's shared memory whose completion bytes go to the
// mbarrier at cluster address `mbar` (the leader's barrier).
__device__ __forceinline__ void tma_load_pair(uint32_t dst, const void* tmap, uint32_t mbar, int32_t x, int32_t y,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(mbar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// One 256 x 256 x 16 MMA of the pair (issued by the leader).
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at this smem offset in both CTAs of the pair once the
// leader's earlier MMAs have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  const uint16_t both = 0x3;
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(smem_u32(bar)),
               "h"(both)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     void* __restrict__ out, int M, int N, int K, int ldd, const ColPlan cp, const RopeArgs rope,
                     const int* __restrict__ groups, int num_groups) {
  static_assert(EPI == kStoreBf16 || EPI == kStoreF32 || EPI == kSwiGLU || EPI == kQkvRope, "plain or QKV epilogues");
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* tfull_bar = empty_bar + kStages;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();     // 0: leader of the pair
  const bool leader = rank == 0;
  const int num_m = (M + kTileM - 1) / kTileM;
  const int num_tiles = num_m * cp.tiles_n;
  const int num_kb = (K + BK - 1) / BK;
  const int pair_id = blockIdx.x / 2;
  const int num_pairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 8);  // one arrival per epilogue warp of both CTAs
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  // the peer's barriers are initialised before any remote arrive or TMA completion
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The weight slabs do not depend on the previous kernel: the first tile's
  // first stages of B go out before the dependency wait (overlapping the
  // previous kernel's tail under programmatic dependent launch); the A loads
  // of those stages follow it.
  const uint64_t pol_b = l2_policy_evict_first();
  const uint32_t full_leader = peer_addr(smem_u32(full_bar), 0);
  int pre = 0;
  // (grouped mode: the group table is the previous kernel's output, so no early loads)
  if (warp == 0 && lane == 0 && pair_id < num_tiles && groups == nullptr) {
    int n0, bn;
    tile_cols(cp, pair_id / num_m, n0, bn);
    const int half = bn / 2;
    n0 += (int)rank * half;
    const uint32_t stage_tx = 2u * (uint32_t)(BM * BK * 2 + half * BK * 2);
    pre = min(kStages, num_kb);
    for (int i = 0; i < pre; ++i) {
      const uint32_t sb = smem_u32(smem + i * kStageBytes) + BM * BK * 2;
      if (leader) mbar_arrive_expect_tx(&full_bar[i], stage_tx);
      for (int b = 0; b < half; b += cp.box_rows)
        tma_load_pair(sb + b * BK * 2, &tmap_b, full_leader + i * 8, i * BK, n0 + b, pol_b);
    }
  }
  pdl_wait();  // everything above touches no memory the previous kernel writes

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool first = true;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        const int m0 = (tile % num_m) * kTileM + (int)rank * BM;
        int n0, bn;
        tile_cols(cp, tile / num_m, n0, bn);
        const int half = bn / 2;                       // B rows this CTA stages
        n0 += (int)rank * half;
        if (groups != nullptr) {                       // the expert of this 256-row tile
          const int g = group_of(groups, num_groups, (tile % num_m) * kTileM);
          if (g < 0) continue;
          n0 += g * N;
        }
        const uint32_t stage_tx = 2u * (uint32_t)(BM * BK * 2 + half * BK * 2);   // both CTAs' bytes
        for (int kb = 0; kb < num_kb; ++kb) {
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + BM * BK * 2;
          const uint32_t fb = full_leader + stage * 8;
          if (!(first && kb < pre)) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, 21)) { ok = false; break; }
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], stage_tx);
            for (int b = 0; b < half; b += cp.box_rows)
              tma_load_pair(sb + b * BK * 2, &tmap_b, fb, kb * BK, n0 + b, pol_b);
          }
          tma_load_pair(sa, &tmap_a, fb, kb * BK, m0, 0ull);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        first = false;
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        // a skipped tile (grouped mode, past the last segment) uses no accumulator
        if (groups != nullptr && group_of(groups, num_groups, (tile % num_m) * kTileM) < 0) continue;
        const int acc = local & 1;
        int n0_unused, bn;
        tile_cols(cp, tile / num_m, n0_unused, bn);
        const uint32_t idesc = idesc_bf16_f32(kTileM, bn);
        if (!mbar_wait(&tempty_bar[acc], ((local >> 1) & 1) ^ 1, 22)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, 23)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + BM * BK * 2;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_pair(d_tmem, sw128_kmajor_desc(sa + kk * 32), sw128_kmajor_desc(sb + kk * 32), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(&empty_bar[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (ok) umma_commit_pair(&tfull_bar[acc]);
        ++local;
      }
    }
  } else {
    const int quad = warp & 3;
    const uint32_t tempty_leader = peer_addr(smem_u32(tempty_bar), 0);
    int local = 0;
    for (int tile = pair_id; tile < num_tiles; tile += num_pairs) {
      if (groups != nullptr && group_of(groups, num_groups, (tile % num_m) * kTileM) < 0) continue;
      const int acc = local & 1;
      ++local;
      if (!mbar_wait(&tfull_bar[acc], ((local - 1) >> 1) & 1, 24)) break;
      tc_fence_after();
      const int m0 = (tile % num_m) * kTileM + (int)rank * BM;
      int n0, bn;
      tile_cols(cp, tile / num_m, n0, bn);
      const int row = m0 + quad * 32 + lane;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * kTileN;
      if constexpr (EPI == kQkvRope) {
        // two whole heads per tile: RoPE on Q / K, K / V into the paged cache
        qkv_rope_row<kTileN>(rope, taddr, row, M, n0, reinterpret_cast<__nv_bfloat16*>(out), ldd);
      } else if constexpr (EPI == kSwiGLU) {
        const int o0 = n0 / 2;
#pragma unroll 1
        for (int c = 0; c < bn / 2; c += 16) {
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
            uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + o0 + c);
            d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < bn; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c, r);
          tmem_wait_ld();
          if (row < M) {
            if constexpr (EPI == kStoreF32) {
              uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<float*>(out) + (size_t)row * ldd + n0 + c);
#pragma unroll
              for (int j = 0; j < 8; ++j) d4[j] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            } else {
              uint32_t packed[16];
#pragma unroll
              for (int j = 0; j < 16; ++j)
                packed[j] = pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
              uint4* d4 =
                  reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + n0 + c);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
            }
          }
        }
      }
      // this warp's TMEM reads are done: one arrival on the leader's barrier
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_leader + acc * 8);
    }
  }

  // Both CTAs finished every MMA, TMEM read and remote arrival before either
  // frees the pair's TMEM or leaves (its shared memory may still be read by
  // the peer's MMAs until then).
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace pair

static int g_pair = -1;

void set_gemm_pair(int on) { g_pair = on ? 1 : 0; }  // declared in gemm_bf16.h

// On by default (it beats the single-CTA kernel on every large shape
// measured); LUNAFLUX_GEMM_2SM=0 turns it off.
static bool pair_enabled() {
  if (g_pair < 0) {
    const char* e = getenv("LUNAFLUX_GEMM_2SM");
    g_pair = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return g_pair == 1;
}

int get_gemm_pair() { return pair_enabled() ? 1 : 0; }  // declared in gemm_bf16.h

// Launches the CTA-pair kernel for large GEMMs (enough 256 x 256 tiles to fill
// the SMs) when it is enabled; returns false otherwise.
static bool run_pair(const GemmArgs& a, int epi, cudaStream_t stream, const RopeArgs& rope = RopeArgs{},
                     const int* groups = nullptr, int num_groups = 0) {
  if (!pair_enabled()) return false;
  if (a.M <= 0 || a.N % pair::kTileN != 0 || a.K % 8 != 0) return false;
  if (epi != kStoreBf16 && epi != kStoreF32 && epi != kSwiGLU && epi != kQkvRope) return false;
  const int sms = num_sms();
  const int tiles = ((a.M + pair::kTileM - 1) / pair::kTileM) * (a.N / pair::kTileN);
  if (tiles < sms / 2) return false;  // skinny shapes keep the split-K kernels
  const int slot = epi == kQkvRope ? 3 : epi;
  auto kfn = epi == kQkvRope ? pair::gemm_pair_kernel<kQkvRope>
             : epi == kSwiGLU ? pair::gemm_pair_kernel<kSwiGLU>
             : (epi == kStoreF32 ? pair::gemm_pair_kernel<kStoreF32> : pair::gemm_pair_kernel<kStoreBf16>);
  static bool attr_set[4] = {false, false, false, false};
  if (!attr_set[slot]) {
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, pair::kSmem);
    attr_set[slot] = true;
  }
  static int max_pairs = 0;
  if (max_pairs == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = pair::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = -1;
    }
    max_pairs = n;
  }
  if (max_pairs < 1) return false;
  pair::ColPlan cp{a.N / pair::kTileN, 0, pair::kTileN, pair::kTileN / 2};
  const int num_m = (a.M + pair::kTileM - 1) / pair::kTileM;
  if (num_m == 1 && epi != kQkvRope && groups == nullptr && a.N % 64 == 0) {
    // one M-tile: k tiles per pair of near-equal width instead of a partial last round
    const int t_min = a.N / pair::kTileN;
    const int k = (t_min + max_pairs - 1) / max_pairs;
    const int t = k * max_pairs;
    const int base = (a.N / (64 * t)) * 64;
    const int wide = base >= 64 ? (a.N - base * t) / 64 : 0;
    if (base >= 64 && base + (wide > 0 ? 64 : 0) <= pair::kTileN && t % max_pairs == 0 && t_min % max_pairs != 0)
      cp = pair::ColPlan{t, wide, base, pair::kBoxRowsNarrow};
  }
  const int all_tiles = num_m * cp.tiles_n;
  const int pairs = all_tiles < max_pairs ? all_tiles : max_pairs;
  CUtensorMap ta = cached_tmap_bf16(a.A, a.M, a.K, a.lda, BM);
  CUtensorMap tb = cached_tmap_bf16(a.B, (uint64_t)a.N * (groups != nullptr ? num_groups : 1), a.K, a.ldb,
                                    (uint32_t)cp.box_rows);
  launch_k(kfn, dim3(2 * pairs), dim3(kThreads), pair::kSmem, stream, 2u, ta, tb, a.D, a.M, a.N, a.K, (int)a.ldd,
           cp, rope, groups, num_groups);
  return true;
}

}  // namespace gemm
}  // namespace lf
