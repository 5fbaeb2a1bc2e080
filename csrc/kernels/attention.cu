// Paged causal GQA attention for sm_100a: decode (one query per row, split-KV)
// and chunked prefill (many queries per row), both reading K/V straight out of
// the paged cache through the block table.
//
// Oracle: kernels/reference/attention.mbt:251-330 in the reference (causal
// GQA, contiguous query-head groups per KV head, scale 1/sqrt(d), max-shifted
// softmax).  The reference's paged operand contract (StepCounts,
// QueryPositions, QueryRowOffsets, SequenceLengths, page table; see
// kernels/launch_contract/README.mbt.md:28-46) maps onto q_start (CSR query
// offsets), seq_lens and a dense per-row block table here.
//
// KV cache layout, per layer and per K/V: [page][kv_head][16 tokens][D=128]
// bf16, so one (page, head) block is 4 KB contiguous.  Pages reach shared
// memory through TMA (2-D tensor map over [pages*heads*16, 128], box 16 x 64,
// 128-byte swizzle; each CTA loads for itself), one mbarrier per stage; fragments come
// out of the swizzled tiles with ldmatrix and feed bf16 mma.sync (m16n8k16).
// Block-table entries are bounds-checked: a bad entry records kErrBadIndex and
// reads the reserved zero page 0 instead.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <unordered_map>

#include "attention.h"
#include "common.cuh"
#include "gemm_bf16.h"

namespace lf {
namespace attn {

constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int kPageBytes = PAGE * D * 2;  // 4 KB: one (page, head) block of K or V

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte offset of (token row r, dim d) inside one page tile loaded as two
// 16x64 boxes with the 128-byte swizzle (d multiple of 8).
__device__ __forceinline__ uint32_t sw_off(int r, int d) {
  const int sub = d >> 6;
  const int chunk = (d & 63) >> 3;
  return sub * 2048 + r * 128 + ((chunk ^ (r & 7)) << 4);
}

// Issue the four TMA boxes of one (page, head): K cols 0-63 / 64-127, V same.
__device__ __forceinline__ void load_page(const CUtensorMap* tk, const CUtensorMap* tv, uint8_t* sk, uint8_t* sv,
                                          uint64_t* bar, int page, int kvh, int Hkv) {
  const int row = (page * Hkv + kvh) * PAGE;
  tma_load_2d(sk, tk, bar, 0, row);
  tma_load_2d(sk + 2048, tk, bar, 64, row);
  tma_load_2d(sv, tv, bar, 0, row);
  tma_load_2d(sv + 2048, tv, bar, 64, row);
}

__device__ __forceinline__ int checked_page(const int32_t* bt, int idx, int num_pages) {
  int p = bt[idx];
  if (p < 0 || p >= num_pages) {
    set_error(kErrBadIndex, (unsigned long long)idx);
    p = 0;
  }
  return p;
}

// Loads the A fragment (16 rows x 16 dims, k-step ks) of Q for rows
// (row0 = lane/4, row1 = lane/4 + 8) whose global pointers are given (null = zero row).
__device__ __forceinline__ void load_q_frag(const __nv_bfloat16* q0, const __nv_bfloat16* q1, int lane,
                                            uint32_t (&a)[8][4]) {
  const int c = 2 * (lane & 3);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int d = ks * 16 + c;
    a[ks][0] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + d) : 0u;
    a[ks][1] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + d) : 0u;
    a[ks][2] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + d + 8) : 0u;
    a[ks][3] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + d + 8) : 0u;
  }
}

// ===========================================================================
// Decode: one warp per (row, kv_head, split).  The warp's 16 MMA rows are the
// G query heads of the KV group (G <= 16; rows >= G are zero).  Pages stream
// through a 4-stage TMA ring owned by the warp.
// ===========================================================================
constexpr int kDecStages = 4;

__global__ void __launch_bounds__(32) decode_kernel(const __grid_constant__ CUtensorMap tk,
                                                    const __grid_constant__ CUtensorMap tv, DecodeArgs a) {
  pdl_trigger();
  // The step's inputs (lengths, token rows, block table) were uploaded before
  // the step's first kernel, and every K / V page except a row's last one was
  // written by earlier steps: the first pages are fetched before the
  // dependency wait (pdl_wait below), the row's last page and Q after it.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecStages * 2 * kPageBytes);
  const int lane = threadIdx.x;
  const int r = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int G = a.Hq / a.Hkv;
  const int L = a.seq_lens[r];
  const int n_pages = (L + PAGE - 1) / PAGE;
  const int pps = (n_pages + a.splits - 1) / a.splits;
  const int p_begin = split * pps;
  const int p_end = min(n_pages, p_begin + pps);
  const int tok = a.tok_index[r];
  const int32_t* bt = a.block_table + (size_t)r * a.bt_stride;

  if (lane == 0) {
    for (int s = 0; s < kDecStages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  const int count = p_end > p_begin ? p_end - p_begin : 0;
  // Block-table window in registers: lane j holds the page of split-relative
  // index win_base + j; the next window is loaded 32 pages ahead of its use,
  // so no refill waits on a block-table read.
  int win_base = 0;
  int win = lane < count ? checked_page(bt, p_begin + lane, a.num_pages) : 0;
  int win_next = 32 + lane < count ? checked_page(bt, p_begin + 32 + lane, a.num_pages) : 0;
  auto page_at = [&](int idx) {  // idx increases monotonically; called by the whole (converged) warp
    while (idx >= win_base + 32) {
      win = win_next;
      win_base += 32;
      const int j = win_base + 32 + lane;
      win_next = j < count ? checked_page(bt, p_begin + j, a.num_pages) : 0;
    }
    return __shfl_sync(0xffffffffu, win, idx - win_base);
  };
  {
    // first pages in flight before Q is read; the row's last page (this
    // step's token) only after the previous kernel has written it
    int first[kDecStages];
#pragma unroll
    for (int i = 0; i < kDecStages; ++i) first[i] = i < count ? page_at(i) : 0;
    const int last = n_pages - 1 - p_begin;   // split-relative index of the row's last page
    if (lane == 0) {
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      for (int i = 0; i < kDecStages && i < count; ++i) {
        if (i == last) continue;
        uint8_t* sk = smem + i * 2 * kPageBytes;
        mbar_arrive_expect_tx(&full[i], 2 * kPageBytes);
        load_page(&tk, &tv, sk, sk + kPageBytes, &full[i], first[i], kvh, a.Hkv);
      }
    }
    pdl_wait();
    if (lane == 0 && last >= 0 && last < kDecStages && last < count) {
      uint8_t* sk = smem + last * 2 * kPageBytes;
      mbar_arrive_expect_tx(&full[last], 2 * kPageBytes);
      load_page(&tk, &tv, sk, sk + kPageBytes, &full[last], first[last], kvh, a.Hkv);
    }
  }

  const int g = lane >> 2;
  const __nv_bfloat16* qbase = a.q + (size_t)tok * a.q_ld + (size_t)kvh * G * D;
  uint32_t qa[8][4];
  load_q_frag(g < G ? qbase + (size_t)g * D : nullptr, g + 8 < G ? qbase + (size_t)(g + 8) * D : nullptr, lane, qa);

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  bool ok = true;
  for (int i = 0; i < count; ++i) {
    const int s = i % kDecStages;
    const uint32_t ph = (i / kDecStages) & 1;
    if (!mbar_wait(&full[s], ph, 10)) { ok = false; break; }
    const uint32_t sk = smem_u32(smem + s * 2 * kPageBytes);
    const uint32_t sv = sk + kPageBytes;
    // S = Q K^T for 16 tokens (two n8 tiles).
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      // x4: m0 = tok 0-7 dims[ks*16, +8), m1 = tok 0-7 dims +8, m2 = tok 8-15 dims, m3 = tok 8-15 dims+8
      const int mi = lane >> 3, rr = lane & 7;
      const int trow = rr + ((mi >> 1) << 3);
      const int dcol = ks * 16 + ((mi & 1) << 3);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(sk + sw_off(trow, dcol), b0, b1, b2, b3);
      mma_bf16(sc[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
      mma_bf16(sc[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
    }
    const int pbase = (p_begin + i) * PAGE;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = pbase + nt * 8 + 2 * (lane & 3) + (e & 1);
        float v = sc[nt][e] * a.scale_log2;
        if (t >= L) v = -INFINITY;
        sc[nt][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float a0 = exp2f(m0 - mx0), a1 = exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][0] = exp2f(sc[nt][0] - mx0);
      sc[nt][1] = exp2f(sc[nt][1] - mx0);
      sc[nt][2] = exp2f(sc[nt][2] - mx1);
      sc[nt][3] = exp2f(sc[nt][3] - mx1);
      ps0 += sc[nt][0] + sc[nt][1];
      ps1 += sc[nt][2] + sc[nt][3];
    }
    l0 = l0 * a0 + ps0;
    l1 = l1 * a1 + ps1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= a0; o[j][1] *= a0; o[j][2] *= a1; o[j][3] *= a1;
    }
    const uint32_t pa0 = pack_bf16x2(sc[0][0], sc[0][1]);
    const uint32_t pa1 = pack_bf16x2(sc[0][2], sc[0][3]);
    const uint32_t pa2 = pack_bf16x2(sc[1][0], sc[1][1]);
    const uint32_t pa3 = pack_bf16x2(sc[1][2], sc[1][3]);
    // O += P V: V tile [16 tok][128 dims]; x4.trans over (tok 0-7, tok 8-15) x (dims n, n+8).
#pragma unroll
    for (int nn = 0; nn < 8; ++nn) {
      const int mi = lane >> 3, rr = lane & 7;
      const int trow = rr + ((mi & 1) << 3);
      const int dcol = nn * 16 + ((mi >> 1) << 3);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(sv + sw_off(trow, dcol), v0, v1, v2, v3);
      mma_bf16(o[2 * nn], pa0, pa1, pa2, pa3, v0, v1);
      mma_bf16(o[2 * nn + 1], pa0, pa1, pa2, pa3, v2, v3);
    }
    __syncwarp();
    if (i + kDecStages < count) {
      const int pg = page_at(i + kDecStages);
      if (lane == 0) {
        fence_proxy_async_smem();
        uint8_t* skp = smem + s * 2 * kPageBytes;
        mbar_arrive_expect_tx(&full[s], 2 * kPageBytes);
        load_page(&tk, &tv, skp, skp + kPageBytes, &full[s], pg, kvh, a.Hkv);
      }
    }
  }
  if (!ok) return;
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int c = 2 * (lane & 3);
  if (a.splits == 1) {
    __nv_bfloat16* ob = a.out + (size_t)tok * a.out_ld + (size_t)kvh * G * D;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (g < G) *reinterpret_cast<uint32_t*>(ob + (size_t)g * D + j * 8 + c) = pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
      if (g + 8 < G)
        *reinterpret_cast<uint32_t*>(ob + (size_t)(g + 8) * D + j * 8 + c) = pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
    }
  } else {
    // Partial results: o normalised by its own l, lse = m + log2(l) (base 2).
    const int h0 = kvh * G + g, h1 = kvh * G + g + 8;
    float* po = a.part_o;
    float* pl = a.part_lse;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (g < G) {
        float* d0 = po + (((size_t)r * a.Hq + h0) * a.splits + split) * D + j * 8 + c;
        d0[0] = o[j][0] * inv0;
        d0[1] = o[j][1] * inv0;
      }
      if (g + 8 < G) {
        float* d1 = po + (((size_t)r * a.Hq + h1) * a.splits + split) * D + j * 8 + c;
        d1[0] = o[j][2] * inv1;
        d1[1] = o[j][3] * inv1;
      }
    }
    if ((lane & 3) == 0) {
      if (g < G) pl[((size_t)r * a.Hq + h0) * a.splits + split] = l0 > 0.f ? m0 + log2f(l0) : -INFINITY;
      if (g + 8 < G) pl[((size_t)r * a.Hq + h1) * a.splits + split] = l1 > 0.f ? m1 + log2f(l1) : -INFINITY;
    }
  }
}

// Merge split-KV partials: out = sum_s w_s * o_s with w_s = 2^(lse_s - lse_max) / sum.
__global__ void decode_combine_kernel(DecodeArgs a) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;  // blockDim = D
  const float* pl = a.part_lse + ((size_t)r * a.Hq + h) * a.splits;
  float mx = -INFINITY;
  for (int s = 0; s < a.splits; ++s) mx = fmaxf(mx, pl[s]);
  float acc = 0.f, wsum = 0.f;
  if (mx > -INFINITY) {
    for (int s = 0; s < a.splits; ++s) {
      const float w = exp2f(pl[s] - mx);
      wsum += w;
      acc += w * a.part_o[(((size_t)r * a.Hq + h) * a.splits + s) * D + d];
    }
  }
  const int tok = a.tok_index[r];
  a.out[(size_t)tok * a.out_ld + (size_t)h * D + d] = __float2bfloat16(wsum > 0.f ? acc / wsum : 0.f);
}

// ===========================================================================
// Prefill: one CTA (4 warps) per (64-query tile, query head, row).  Each warp
// owns 16 queries; K/V tiles of 64 tokens (4 pages) stream through a 2-stage
// TMA ring shared by the 4 warps.
// ===========================================================================
constexpr int kPreStages = 2;
constexpr int kTileTok = 64;
constexpr int kTileBytes = 4 * kPageBytes;  // 16 KB of K (or V) per tile

__global__ void __launch_bounds__(128) prefill_kernel(const __grid_constant__ CUtensorMap tk,
                                                      const __grid_constant__ CUtensorMap tv, PrefillArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPreStages * 2 * kTileBytes);
  uint64_t* empty = full + kPreStages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.z, h = blockIdx.y;
  const int G = a.Hq / a.Hkv;
  const int kvh = h / G;
  const int qs = a.q_start[r];
  const int ql = a.q_start[r + 1] - qs;
  const int q0 = blockIdx.x * 64;
  if (q0 >= ql) return;
  const int L = a.seq_lens[r];
  const int ctx = L - ql;  // absolute position of the row's first query
  const int n_pages_row = (L + PAGE - 1) / PAGE;
  const int block_last_pos = ctx + min(q0 + 64, ql) - 1;
  const int n_tiles = block_last_pos / kTileTok + 1;
  const int32_t* bt = a.block_table + (size_t)r * a.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPreStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int tile, int s) {
    uint8_t* sk = smem + s * 2 * kTileBytes;
    uint8_t* sv = sk + kTileBytes;
    mbar_arrive_expect_tx(&full[s], 2 * kTileBytes);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int pi = tile * 4 + j;
      const int page = pi < n_pages_row ? checked_page(bt, pi, a.num_pages) : 0;
      load_page(&tk, &tv, sk + j * kPageBytes, sv + j * kPageBytes, &full[s], page, kvh, a.Hkv);
    }
  };
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    for (int i = 0; i < kPreStages && i < n_tiles; ++i) issue(i, i);
  }

  const int g = lane >> 2;
  const int qw = q0 + warp * 16;  // first query (chunk-relative) of this warp
  const int qrow0 = qw + g, qrow1 = qw + g + 8;
  const __nv_bfloat16* qp0 = qrow0 < ql ? a.q + (size_t)(qs + qrow0) * a.q_ld + (size_t)h * D : nullptr;
  const __nv_bfloat16* qp1 = qrow1 < ql ? a.q + (size_t)(qs + qrow1) * a.q_ld + (size_t)h * D : nullptr;
  uint32_t qa[8][4];
  load_q_frag(qp0, qp1, lane, qa);
  const int pos0 = ctx + qrow0, pos1 = ctx + qrow1;
  const int warp_last_pos = ctx + min(qw + 15, ql - 1);
  const bool warp_active = qw < ql;

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool ok = true;

  for (int i = 0; i < n_tiles; ++i) {
    const int s = i % kPreStages;
    const uint32_t ph = (i / kPreStages) & 1;
    if (!mbar_wait(&full[s], ph, 20)) { ok = false; break; }
    const int tbase = i * kTileTok;
    if (warp_active && tbase <= warp_last_pos) {
      const uint32_t sk = smem_u32(smem + s * 2 * kTileBytes);
      const uint32_t sv = sk + kTileBytes;
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int pg = 0; pg < 4; ++pg) {
          const int mi = lane >> 3, rr = lane & 7;
          const int trow = rr + ((mi >> 1) << 3);
          const int dcol = ks * 16 + ((mi & 1) << 3);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sk + pg * kPageBytes + sw_off(trow, dcol), b0, b1, b2, b3);
          mma_bf16(sc[2 * pg], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
          mma_bf16(sc[2 * pg + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
        }
      }
      float mx0 = m0, mx1 = m1;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = tbase + nt * 8 + 2 * (lane & 3) + (e & 1);
          const int qpos = e < 2 ? pos0 : pos1;
          float v = sc[nt][e] * a.scale_log2;
          if (t > qpos) v = -INFINITY;
          sc[nt][e] = v;
        }
        mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      // Rows whose queries are all masked so far keep m = -inf; use 0 as the
      // shift so exp2 never sees (-inf) - (-inf).
      const float sh0 = mx0 == -INFINITY ? 0.f : mx0;
      const float sh1 = mx1 == -INFINITY ? 0.f : mx1;
      const float a0 = exp2f(m0 - sh0), a1 = exp2f(m1 - sh1);
      m0 = mx0;
      m1 = mx1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        sc[nt][0] = exp2f(sc[nt][0] - sh0);
        sc[nt][1] = exp2f(sc[nt][1] - sh0);
        sc[nt][2] = exp2f(sc[nt][2] - sh1);
        sc[nt][3] = exp2f(sc[nt][3] - sh1);
        ps0 += sc[nt][0] + sc[nt][1];
        ps1 += sc[nt][2] + sc[nt][3];
      }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= a0; o[j][1] *= a0; o[j][2] *= a1; o[j][3] *= a1;
      }
#pragma unroll
      for (int pg = 0; pg < 4; ++pg) {
        const uint32_t pa0 = pack_bf16x2(sc[2 * pg][0], sc[2 * pg][1]);
        const uint32_t pa1 = pack_bf16x2(sc[2 * pg][2], sc[2 * pg][3]);
        const uint32_t pa2 = pack_bf16x2(sc[2 * pg + 1][0], sc[2 * pg + 1][1]);
        const uint32_t pa3 = pack_bf16x2(sc[2 * pg + 1][2], sc[2 * pg + 1][3]);
#pragma unroll
        for (int nn = 0; nn < 8; ++nn) {
          const int mi = lane >> 3, rr = lane & 7;
          const int trow = rr + ((mi & 1) << 3);
          const int dcol = nn * 16 + ((mi >> 1) << 3);
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(sv + pg * kPageBytes + sw_off(trow, dcol), v0, v1, v2, v3);
          mma_bf16(o[2 * nn], pa0, pa1, pa2, pa3, v0, v1);
          mma_bf16(o[2 * nn + 1], pa0, pa1, pa2, pa3, v2, v3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (threadIdx.x == 0 && i + kPreStages < n_tiles) {
      if (!mbar_wait(&empty[s], ph, 21)) { ok = false; break; }
      fence_proxy_async_smem();
      issue(i + kPreStages, s);
    }
  }
  if (!ok || !warp_active) return;
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int c = 2 * (lane & 3);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (qrow0 < ql)
      *reinterpret_cast<uint32_t*>(a.out + (size_t)(qs + qrow0) * a.out_ld + (size_t)h * D + j * 8 + c) =
          pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    if (qrow1 < ql)
      *reinterpret_cast<uint32_t*>(a.out + (size_t)(qs + qrow1) * a.out_ld + (size_t)h * D + j * 8 + c) =
          pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace {
std::mutex g_mu;
std::unordered_map<const void*, std::pair<uint64_t, CUtensorMap>> g_maps;
}  // namespace

static CUtensorMap cache_map(const void* base, int64_t rows) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_maps.find(base);
  if (it != g_maps.end() && it->second.first == (uint64_t)rows) return it->second.second;
  CUtensorMap m = gemm::make_tmap_2d(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, D, D, PAGE, 64,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  g_maps[base] = {(uint64_t)rows, m};
  return m;
}

// Decode CTAs (one warp each) resident per SM, from the kernel's resources.
static int decode_ctas_per_sm() {
  static int n = 0;
  if (n == 0) {
    const int smem = kDecStages * 2 * kPageBytes + 1024 + 64;
    cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel, 32, smem) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = 6;
    }
  }
  return n;
}

// Split-KV count: the fewest splits that give about half of the resident CTA
// slots (num_sms x ctas_per_sm) work, with at least 8 pages per split and at
// most 32 splits.  Measured on B200 (one warp per CTA, 6 per SM): 256 rows x
// 8 heads x 72 pages and 64 x 8 x 128 run fastest unsplit (2048 and 512
// CTAs), 128 rows x 1 head x 144 pages with 4 splits, 1 row x 8 heads x 256
// pages with 16 or more; splitting a grid that already fills the slots only
// adds the combine pass.
int decode_splits(int rows, int Hkv, int max_seq, int num_sms) {
  const int units = rows * Hkv;
  const int pages = (max_seq + PAGE - 1) / PAGE;
  if (units <= 0 || pages <= 0) return 1;
  const int64_t half_slots = (int64_t)num_sms * decode_ctas_per_sm() / 2;
  int s = (int)((half_slots + units - 1) / units);
  if (s > 32) s = 32;
  while (s > 1 && pages / s < 8) --s;
  return s < 1 ? 1 : s;
}

void decode(const DecodeArgs& a_in, const void* kcache, const void* vcache, cudaStream_t stream) {
  DecodeArgs a = a_in;
  if (a.rows <= 0) return;
  if (a.D != D || a.page != PAGE) throw std::runtime_error("lunaflux attention: head_dim 128 and page 16 only");
  if (a.Hq % a.Hkv != 0 || a.Hq / a.Hkv > 16) throw std::runtime_error("lunaflux attention: GQA group must be <= 16");
  const int64_t rows = (int64_t)a.num_pages * a.Hkv * PAGE;
  CUtensorMap tk = cache_map(kcache, rows), tv = cache_map(vcache, rows);
  const int smem = kDecStages * 2 * kPageBytes + 1024 + 64;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  if (a.splits > 1 && (a.part_o == nullptr || a.part_lse == nullptr))
    throw std::runtime_error("lunaflux attention: split-KV decode needs a workspace");
  dim3 grid(a.rows, a.Hkv, a.splits);
  launch_k(decode_kernel, dim3(grid), dim3(32), smem, stream, 1,
         tk, tv, a);
  if (a.splits > 1) launch_k(decode_combine_kernel, dim3(dim3(a.rows, a.Hq)), dim3(D), 0, stream, 1,
         a);
}

void prefill(const PrefillArgs& a, const void* kcache, const void* vcache, cudaStream_t stream) {
  if (a.rows <= 0 || a.max_q_len <= 0) return;
  if (a.D != D || a.page != PAGE) throw std::runtime_error("lunaflux attention: head_dim 128 and page 16 only");
  const int64_t rows = (int64_t)a.num_pages * a.Hkv * PAGE;
  CUtensorMap tk = cache_map(kcache, rows), tv = cache_map(vcache, rows);
  // The tcgen05 kernel for supported GQA groups; LUNAFLUX_PREFILL_MMA_SYNC
  // selects the mma.sync kernel instead (for comparison).
  if (prefill_tc_supported(a) && std::getenv("LUNAFLUX_PREFILL_MMA_SYNC") == nullptr) {
    prefill_tc(a, tk, tv, stream);
    return;
  }
  const int smem = kPreStages * 2 * kTileBytes + 1024 + 64;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  dim3 grid((a.max_q_len + 63) / 64, a.Hq, a.rows);
  prefill_kernel<<<grid, 128, smem, stream>>>(tk, tv, a);
}

}  // namespace attn
}  // namespace lf
