// Paged causal GQA prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), for chunked prefill.
//
// Oracle: kernels/reference/attention.mbt:251-330 in the reference (causal
// GQA, scale 1/sqrt(d), max-shifted softmax); operands as in attention.cu
// (CSR query offsets, sequence lengths, dense block table, KV layout
// [page][kv_head][16][128]).
//
// One CTA = one (row, KV head, query tile).  The tile's 128 MMA rows are the
// G = Hq / Hkv query heads of the KV head times 128 / G query tokens (head
// major), so every K/V block is staged once for the whole GQA group.  Per
// 128-key block j:
//
//   S_j  = Q . K_j^T          tcgen05.mma, Q and K_j K-major in shared memory,
//                             S in TMEM (double-buffered, so S_{j+1} is
//                             computed while the softmax works on S_j)
//   P_j  = exp2(S_j - m)      8 softmax warps, two per TMEM lane quadrant: a
//                             row (TMEM lane) is shared by two threads, each
//                             taking 64 of its 128 scores; the halves swap
//                             their partial maxima through shared memory.
//                             P written to shared memory (bf16, 128-byte
//                             swizzle, double-buffered, so the softmax of
//                             block j+1 overlaps the P.V MMA of block j)
//   O   += P_j . V_j          tcgen05.mma, V_j MN-major (the page layout
//                             itself), O in TMEM
//
// The running maximum used for P only moves when a row maximum grows by more
// than 8 (in log2 units): then O and the row sums of the warp are rescaled
// through TMEM (warp-uniformly: tcgen05.ld / st are warp-collective).
// Between such events P may exceed 1 by at most 2^8, well inside fp32 and
// bf16 range; the final O / l is unchanged.
//
// Warp roles (320 threads): warp 0 lane 0 issues the TMA loads (Q once, then
// K and V pages of each block into a 2-stage ring), warp 1 owns TMEM and its
// lane 0 issues the MMAs, warps 2..9 run the softmax and the epilogue (warps
// w and w + 4 share the TMEM lanes of quadrant w % 4: columns 0..63 and
// 64..127 of S, P and O).  All
// waits are bounded (common.cuh); every TMA load fills only its own CTA.
// Block-table entries are bounds-checked (kErrBadIndex, zero page instead).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <stdexcept>
#include <tuple>
#include <unordered_map>

#include "attention.h"
#include "common.cuh"
#include "gemm_bf16.h"

namespace lf {
namespace attn {
namespace tc {

constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int KB = 128;                    // keys per block
constexpr int kTile = 128 * 128 * 2;       // one 128 x 128 bf16 operand tile, 32 KB
constexpr int kHalf = kTile / 2;           // its 64-column half (16 KB)
// shared memory: Q | K[2] | V[2] | P[2] | barriers  (224 KB + barriers)
constexpr int kOffQ = 0;
constexpr int kOffK = kTile;
constexpr int kOffV = 3 * kTile;
constexpr int kOffP = 5 * kTile;
constexpr int kOffBar = 7 * kTile;
constexpr int kOffRed = kOffBar + 256;     // [2 halves][128 rows] fp32: partial row maxima / sums
constexpr int kOffFlag = kOffRed + 1024;   // [2 halves][4 quadrants] int: the warp's pipeline is sound
constexpr int kSmem = 7 * kTile + 256 + 1024 + 1024 + 64;
constexpr int kThreadsTc = 320;
constexpr uint32_t kColsS0 = 0, kColsS1 = 128, kColsO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;   // sm_100 descriptor version
  d |= (uint64_t)2 << 61;   // 128-byte swizzle
  return d;
}
// K-major operand [rows][128] stored as two 64-column halves of [rows][128 B]:
// k-step kk (16 columns) starts in half kk / 4 at byte (kk % 4) * 32.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return smem_desc(base + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}
// MN-major operand (V: [keys][128 dims], dims contiguous): k-step kk covers
// keys 16 kk .. 16 kk + 15 (2 KB further on); the two 64-dim halves are 16 KB
// apart (leading byte offset), 8-key groups 1 KB apart (stride byte offset).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk) {
  return smem_desc(base + kk * 2048, kHalf, 1024);
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 2^x with the hardware's approximate base-2 exponential (ex2.approx.ftz: a
// few ulp; -inf -> +0), the same instruction the fast exp paths use.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void bar_sync_n(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Diagnostics, compiled in only with -DLF_ATTN_PROGRESS_TRACE: the CTA's
// progress code, written through to host-visible memory (PrefillArgs.progress).
__device__ __forceinline__ void mark(const PrefillArgs& a, int code) {
#ifdef LF_ATTN_PROGRESS_TRACE
  if (a.progress != nullptr) {
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(a.progress + cta), "r"(code) : "memory");
  }
#else
  (void)a;
  (void)code;
#endif
}

__device__ __forceinline__ int bt_page(const PrefillArgs& a, int r, int idx) {
  int p = a.block_table[(int64_t)r * a.bt_stride + idx];
  if (p < 0 || p >= a.num_pages) {
    set_error(kErrBadIndex, (unsigned long long)idx);
    p = 0;
  }
  return p;
}

// One work item: (query tile qb, row r, KV head h).  Items are numbered
// longest tile first; an item whose tile starts past the row's queries is empty.
struct Item {
  bool live;
  int r, h, qs, n, t0, pos0, kmax, nkb;
};

__device__ __forceinline__ Item item_of(const PrefillArgs& a, int w, int nq, int QT) {
  Item it;
  const int per = a.rows * a.Hkv;
  const int qb = nq - 1 - w / per;
  const int rem = w % per;
  it.r = rem / a.Hkv;
  it.h = rem % a.Hkv;
  it.qs = a.q_start[it.r];
  it.n = a.q_start[it.r + 1] - it.qs;
  it.t0 = qb * QT;
  it.live = it.t0 < it.n;
  const int L = a.seq_lens[it.r];
  it.pos0 = L - it.n;                                   // position of the row's first query
  it.kmax = it.pos0 + min(it.n, it.t0 + QT) - 1;        // last key any query of the tile sees
  it.nkb = it.live ? it.kmax / KB + 1 : 0;
  return it;
}

// Persistent: CTA c takes items c, c + gridDim.x, ...  The K / V ring, the S
// buffers and the P buffers are indexed by a block counter that runs across
// the CTA's items, so the next item's Q, K and V loads and its first S MMA
// overlap the previous item's last softmax and epilogue.  Q is reloaded once
// the previous item's last S MMA is done (q_empty); the first P . V of an item
// overwrites O only after the softmax warps have read the previous item's O
// (o_empty).
__global__ void __launch_bounds__(kThreadsTc, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tq,
                                                            const __grid_constant__ CUtensorMap tk,
                                                            const __grid_constant__ CUtensorMap tv, PrefillArgs a,
                                                            int G, int nq) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* k_empty = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;    // [2]
  uint64_t* s_full = bars + 9;     // [2]
  uint64_t* s_empty = bars + 11;   // [2]
  uint64_t* p_full = bars + 13;    // [2] per P buffer
  uint64_t* pv_done = bars + 15;   // [2] per P buffer: P . V of that buffer's block done
  uint64_t* q_empty = bars + 17;   // the item's last S MMA is done: Q may be reloaded
  uint64_t* o_empty = bars + 18;   // the softmax warps have read the item's O
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int QT = 128 / G;                         // query tokens per tile
  const int W = nq * a.rows * a.Hkv;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(o_empty, 256);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 256);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&p_full[b], 256);
      mbar_init(&pv_done[b], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      int gb = 0, ni = 0;   // blocks and items this CTA has loaded
      for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
        const Item it = item_of(a, w, nq, QT);
        if (!it.live) continue;
        // Q: G heads x QT tokens, each a [QT][64] box per 64-column half
        if (!mbar_wait(q_empty, (ni & 1) ^ 1, 20)) break;
        mbar_arrive_expect_tx(q_full, kTile);
        for (int g = 0; g < G; ++g)
          for (int half = 0; half < 2; ++half)
            tma_load_2d(smem + kOffQ + half * kHalf + g * QT * 128, &tq, q_full, (it.h * G + g) * D + half * 64,
                        it.qs + it.t0);
        ++ni;
        for (int j = 0; j < it.nkb; ++j, ++gb) {
          const int s = gb & 1;
          const uint32_t ph = ((gb >> 1) & 1) ^ 1;
          int pages[8];
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int idx = j * 8 + p;
            pages[p] = idx * PAGE <= it.kmax ? bt_page(a, it.r, idx) : 0;   // past the last key: the zero page
          }
          if (!mbar_wait(&k_empty[s], ph, 21)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[s], kTile);
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int row = (pages[p] * a.Hkv + it.h) * PAGE;
            uint8_t* dst = smem + kOffK + s * kTile + p * 2048;
            tma_load_2d(dst, &tk, &k_full[s], 0, row);
            tma_load_2d(dst + kHalf, &tk, &k_full[s], 64, row);
          }
          if (!mbar_wait(&v_empty[s], ph, 22)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[s], kTile);
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int row = (pages[p] * a.Hkv + it.h) * PAGE;
            uint8_t* dst = smem + kOffV + s * kTile + p * 2048;
            tma_load_2d(dst, &tv, &v_full[s], 0, row);
            tma_load_2d(dst + kHalf, &tv, &v_full[s], 64, row);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128);              // Q . K^T, both K-major
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128) | (1u << 16); // P . V, V MN-major
      bool ok = true;
      int gb = 0, ni = 0;
      auto issue_s = [&](int g) -> bool {
        const int s = g & 1;
        if (!mbar_wait(&k_full[s], (g >> 1) & 1, 24)) return false;
        if (!mbar_wait(&s_empty[s], ((g >> 1) & 1) ^ 1, 25)) return false;
        tc_fence_after();
        const uint32_t dS = tmem + (s ? kColsS1 : kColsS0);
        const uint32_t qa = sbase + kOffQ, kb = sbase + kOffK + s * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16_ss(dS, kmajor_desc(qa, kk), kmajor_desc(kb, kk), idesc_s, kk > 0);
        // the stage release first, the barrier someone waits on last: commits
        // land in issue order, so no arrive is still in flight once the
        // waiter has seen the last one (a CTA must not exit under a pending
        // arrive on its shared memory)
        umma_commit(&k_empty[s]);
        umma_commit(&s_full[s]);
        return true;
      };
      for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
        const Item it = item_of(a, w, nq, QT);
        if (!it.live) continue;
        if (!mbar_wait(q_full, ni & 1, 23)) break;
        tc_fence_after();
        if (!issue_s(gb)) break;
        if (it.nkb == 1) umma_commit(q_empty);
        for (int j = 0; j < it.nkb; ++j) {
          const int g = gb + j;
          if (j + 1 < it.nkb) {
            if (!issue_s(g + 1)) { ok = false; break; }
            if (j + 2 == it.nkb) umma_commit(q_empty);    // the item's last S MMA has been issued
          }
          const int s = g & 1;
          if (!mbar_wait(&p_full[s], (g >> 1) & 1, 26) || !mbar_wait(&v_full[s], (g >> 1) & 1, 27)) {
            ok = false;
            break;
          }
          // the first P . V of an item overwrites O: the previous item's O has been read
          if (j == 0 && !mbar_wait(o_empty, (ni & 1) ^ 1, 28)) { ok = false; break; }
          tc_fence_after();
          const uint32_t pa = sbase + kOffP + s * kTile, vb = sbase + kOffV + s * kTile;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16_ss(tmem + kColsO, kmajor_desc(pa, kk), mnmajor_desc(vb, kk), idesc_o, (j > 0 || kk > 0));
          umma_commit(&v_empty[s]);
          umma_commit(&pv_done[s]);
        }
        gb += it.nkb;
        ++ni;
      }
    }
  } else {
    // softmax + epilogue: warp w reads TMEM lanes of quadrant w % 4; warps
    // 2..5 take columns 0..63 of their rows, warps 6..9 columns 64..127
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int c0 = half * 64;
    const int row = quad * 32 + lane;
    const int g = row / QT, t = row % QT;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = a.scale_log2;
    float* red = reinterpret_cast<float*>(smem + kOffRed);   // [2][128]
    volatile int* flag = reinterpret_cast<volatile int*>(smem + kOffFlag);   // [2][4]
    const int bar_id = 1 + quad;                             // the two warps of this quadrant
    uint8_t* prow0 = smem + kOffP + half * kHalf + row * 128;
    bool ok = true;
    int gb = 0;
    for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
      const Item it = item_of(a, w, nq, QT);
      if (!it.live) continue;
      const int tok = it.t0 + t;
      const bool valid = tok < it.n;
      const int pos = it.pos0 + tok;
      const int nkb = it.nkb;
      float m_used = -INFINITY, l = 0.f;
      // The two warps of a quadrant meet at named barriers twice per block.  A
      // failed (timed-out) wait never makes one of them leave alone: it only
      // marks the warp unsound, both warps publish their state at the next
      // exchange and leave the loop there together, so neither is left at a
      // barrier the other will not reach.
      for (int j = 0; j < nkb; ++j) {
        const int gj = gb + j;
        const int s = gj & 1;
        // every wait before a warp-collective TMEM access is made warp-uniform:
        // tcgen05.ld / st are .sync.aligned and must not run in a diverged warp
        if (ok && !__all_sync(0xffffffffu, mbar_wait(&s_full[s], (gj >> 1) & 1, 28))) ok = false;
        float x[64];
        float pm = -INFINITY;
        if (ok) {
          tc_fence_after();
          // this thread's 64 scores of its row: two TMEM loads in flight, one wait
          uint32_t v0[32], v1[32];
          const uint32_t srow = tmem + lane_off + (s ? kColsS1 : kColsS0) + c0;
          tmem_ld_32x32b_x32(srow, v0);
          tmem_ld_32x32b_x32(srow + 32, v1);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            x[e] = __uint_as_float(v0[e]);
            x[32 + e] = __uint_as_float(v1[e]);
          }
          tc_fence_before();
          mbar_arrive(&s_empty[s]);     // the MMA warp may compute S_{j+2} into this buffer
          // row maximum of the raw scores (scale > 0 commutes with max); the
          // mask is applied only on blocks that cross this row's causal limit
          const int key0 = j * KB + c0;
          float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          if (valid && key0 + 63 <= pos) {
#pragma unroll
            for (int c = 0; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], x[c]);
          } else {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              if (!valid || key0 + c > pos) x[c] = -INFINITY;
              m4[c & 3] = fmaxf(m4[c & 3], x[c]);
            }
          }
          pm = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        }
        // the row maximum over both halves, and both warps' state, through shared memory
        red[half * 128 + row] = pm;
        if (lane == 0) flag[half * 4 + quad] = ok ? 1 : 0;
        bar_sync_n(bar_id, 64);
        const bool both_ok = flag[quad] != 0 && flag[4 + quad] != 0;
        const float mx = fmaxf(red[row], red[128 + row]) * sl2;   // log2 units
        bar_sync_n(bar_id, 64);                                   // both read before the next write
        if (!both_ok) {
          ok = false;
          break;
        }
        // P buffer gj % 2 is free once P . V of block gj - 2 is done (that block
        // may belong to the previous item); a rescale of O also needs P . V of
        // this item's previous block done
        if (gj > 1 && !__all_sync(0xffffffffu, mbar_wait(&pv_done[s], ((gj >> 1) & 1) ^ 1, 29))) {
          ok = false;
          continue;   // leave together with the partner warp at the next exchange
        }
        uint8_t* prow = prow0 + s * kTile;
        // The rescale touches O through TMEM with warp-collective instructions,
        // so the whole warp rescales when any of its rows needs to; both warps
        // of a quadrant hold the same rows and the same maxima, so they decide
        // alike, and rows whose maximum moved less rescale by their own factor.
        if (__any_sync(0xffffffffu, mx > m_used + kRescaleThreshold)) {
          if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&pv_done[s ^ 1], ((gj - 1) >> 1) & 1, 31))) {
            ok = false;
            continue;
          }
          const float m_new = fmaxf(m_used, mx);
          const float alpha = m_used == -INFINITY ? (m_new == -INFINITY ? 1.f : 0.f) : ex2_approx(m_used - m_new);
          if (j > 0) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 64; c += 32) {
              uint32_t v[32];
              tmem_ld_32x32b_x32(tmem + lane_off + kColsO + c0 + c, v);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
              tmem_st_32x32b_x32(tmem + lane_off + kColsO + c0 + c, v);
            }
            tmem_wait_st();
          }
          l *= alpha;
          m_used = m_new;
        }
        // P = exp2(s * scale_log2 - m) as bf16 into this half of the swizzled
        // [key-half][row][128 B] tile
        const float neg_m = m_used == -INFINITY ? 0.f : -m_used;   // all-masked row: every p is 0
        float l2[2] = {0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = ex2_approx(fmaf(x[c + 2 * e], sl2, neg_m));
            const float p1 = ex2_approx(fmaf(x[c + 2 * e + 1], sl2, neg_m));
            l2[0] += p0;
            l2[1] += p1;
            wv[e] = pack_bf16x2(p0, p1);
          }
          const int chunk = c >> 3;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (row & 7)) << 4)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        l += l2[0] + l2[1];
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[s]);
      }
      // O is complete once P . V of the item's last block is done.  That wait,
      // too, can only fail: its outcome and the row sum are exchanged with the
      // partner warp, and both act on the joint state (both write the item's
      // output and go on, or both leave), so neither is ever left alone at a
      // named barrier of the next item.
      const int gl = gb + nkb - 1;
      if (ok && !__all_sync(0xffffffffu, mbar_wait(&pv_done[gl & 1], (gl >> 1) & 1, 30))) ok = false;
      red[half * 128 + row] = l;
      if (lane == 0) flag[half * 4 + quad] = ok ? 1 : 0;
      bar_sync_n(bar_id, 64);
      const float l_row = red[row] + red[128 + row];
      ok = flag[quad] != 0 && flag[4 + quad] != 0;
      bar_sync_n(bar_id, 64);                                     // both read before the next item's writes
      if (ok) {
        tc_fence_after();
        const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
        __nv_bfloat16* dst = a.out + (int64_t)(it.qs + tok) * a.out_ld + (it.h * G + g) * D + c0;
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + lane_off + kColsO + c0 + c, v);
          tmem_wait_ld();
          if (valid) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              pk[e] = pack_bf16x2(__uint_as_float(v[2 * e]) * inv, __uint_as_float(v[2 * e + 1]) * inv);
            uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
            for (int e = 0; e < 4; ++e) d4[e] = make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(o_empty);          // the next item's first P . V may overwrite O
      }
      gb += nkb;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

static std::mutex g_mu;
static std::unordered_map<std::string, CUtensorMap> g_q;

static CUtensorMap q_map(const PrefillArgs& a, int qt) {
  const std::string key = std::to_string((uintptr_t)a.q) + ":" + std::to_string(a.q_rows) + ":" +
                          std::to_string(a.q_ld) + ":" + std::to_string(a.Hq) + ":" + std::to_string(qt);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_q.find(key);
  if (it != g_q.end()) return it->second;
  CUtensorMap m = gemm::make_tmap_2d(a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.q_rows, (uint64_t)a.Hq * D, a.q_ld,
                                     qt, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (g_q.size() > 256) g_q.clear();
  g_q[key] = m;
  return m;
}

}  // namespace tc

bool prefill_tc_supported(const PrefillArgs& a) {
  if (a.D != tc::D || a.page != tc::PAGE || a.Hkv <= 0 || a.Hq % a.Hkv != 0 || a.q_rows <= 0) return false;
  const int G = a.Hq / a.Hkv;
  return G == 1 || G == 2 || G == 4 || G == 8 || G == 16;
}

void prefill_tc(const PrefillArgs& a, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
  const int G = a.Hq / a.Hkv;
  const int QT = 128 / G;
  CUtensorMap tq = tc::q_map(a, QT);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(tc::prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem);
    attr = true;
  }
  const int nq = (a.max_q_len + QT - 1) / QT;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int items = nq * a.rows * a.Hkv;
  const int grid = items < sms ? items : sms;   // persistent: one CTA per SM (224 KB of shared memory)
  launch_k(tc::prefill_tc_kernel, dim3(grid), dim3(tc::kThreadsTc), tc::kSmem, stream, 1, tq, tk, tv, a, G, nq);
}

}  // namespace attn
}  // namespace lf
