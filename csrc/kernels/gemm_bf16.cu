// Persistent warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05 + TMEM), operands staged by TMA.
//
//   D[M, N] = A[M, K] . B[N, K]^T      (A: activations, B: weight [out, in])
//
// This is the projection primitive behind every linear layer of the model
// (QKV, o_proj, gate/up, down, LM head).  The reference only plans these as
// external AOT modules or a cuBLASLt call (internal/cuda/gemm.c:108-207 in the
// reference); here it is a hand-written Blackwell kernel.
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer: A and B k-slabs (64 bf16 = 128 B wide, 128-byte
//               swizzle) into a STAGES-deep shared-memory ring.
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN, K=16)
//               into one of two TMEM accumulators and commits to mbarriers.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (each warp owns the 32
//               TMEM lanes of its quadrant), convert, store; the second TMEM
//               accumulator lets the next tile's MMAs overlap this epilogue.
//
// Epilogues: plain bf16 store, fp32 store (LM-head logits), and SwiGLU over a
// gate/up weight whose rows are interleaved in groups of 64 (32 gate rows, then
// the 32 up rows of the same features): the gate/up projection writes
// silu(gate) * up directly and the [M, 2F] intermediate never exists.
//
// All waits are bounded (common.cuh); no TMA load uses cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "gemm_bf16.h"

namespace lf {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;                 // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

enum Epi : int { kStoreBf16 = 0, kStoreF32 = 1, kSwiGLU = 2, kSplitF32 = 3 };

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

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b, void* __restrict__ out, int M,
                     int N, int K, int ldd, int splits, int kb_per_split) {
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
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, 1)) { ok = false; break; }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full_bar[stage], S::kStageBytes);
          tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * BK, m0);
          tma_load_2d_hint(sb, &tmap_b, &full_bar[stage], kb * BK, n0, pol_b);
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
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + n0 + c;
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kCols);
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

// ---------------------------------------------------------------------------
// Host side: tensor maps and launch.
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      throw std::runtime_error("lunaflux: cuTensorMapEncodeTiled is unavailable");
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                         uint64_t cols, uint64_t ld_elems, uint32_t box_rows, uint32_t box_cols,
                         CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (strides[0] & 15) != 0) {
    throw std::runtime_error("lunaflux: TMA operand must be 16-byte aligned with a 16-byte row stride");
  }
  CUresult r = get_encode_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    throw std::runtime_error("lunaflux: cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  }
  return m;
}

namespace {
struct TmapKey {
  const void* p;
  uint64_t rows, cols, ld;
  uint32_t box_rows;
  bool operator==(const TmapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    size_t h = std::hash<const void*>()(k.p);
    h ^= std::hash<uint64_t>()(k.rows * 1000003ull + k.cols) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<uint64_t>()(k.ld * 31ull + k.box_rows) + (h << 6) + (h >> 2);
    return h;
  }
};
std::mutex g_tmap_mu;
std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> g_tmap_cache;
}  // namespace

static CUtensorMap cached_tmap_bf16(const void* p, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  TmapKey k{p, rows, cols, ld, box_rows};
  std::lock_guard<std::mutex> g(g_tmap_mu);
  auto it = g_tmap_cache.find(k);
  if (it != g_tmap_cache.end()) return it->second;
  if (g_tmap_cache.size() > 65536) g_tmap_cache.clear();
  CUtensorMap m = make_tmap_2d(p, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, ld, box_rows, BK,
                               CU_TENSOR_MAP_SWIZZLE_128B);
  g_tmap_cache.emplace(k, m);
  return m;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int STAGES, int EPI>
static void launch(const GemmArgs& a, cudaStream_t stream, int splits = 1, int kb_per = 0, float* ws = nullptr) {
  using S = Smem<BN, STAGES>;
  auto kfn = gemm_bf16_kernel<BN, STAGES, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    attr_set = true;
  }
  CUtensorMap ta = cached_tmap_bf16(a.A, a.M, a.K, a.lda, BM);
  CUtensorMap tb = cached_tmap_bf16(a.B, a.N, a.K, a.ldb, BN);
  const int tiles = ((a.M + BM - 1) / BM) * (a.N / BN) * splits;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  if (kb_per <= 0) kb_per = (a.K + BK - 1) / BK;
  if (EPI == kSplitF32) {
    kfn<<<grid, kThreads, S::kTotal, stream>>>(ta, tb, ws, a.M, a.N, a.K, a.N, splits, kb_per);
  } else {
    kfn<<<grid, kThreads, S::kTotal, stream>>>(ta, tb, a.D, a.M, a.N, a.K, a.ldd, splits, kb_per);
  }
}

// Split-K plan for skinny GEMMs: 256-wide tiles (so the activations are
// re-read from L2 as few times as possible) and enough K-splits to cover the
// SMs, each split at least 4 k-blocks.  Returns splits (1 = no split).
int plan_splitk(int M, int N, int K, int* kb_per_out) {
  const int sms = num_sms();
  const int num_m = (M + BM - 1) / BM;
  const int num_kb = (K + BK - 1) / BK;
  if (N % 256 != 0) return 1;
  const int tiles = num_m * (N / 256);
  if (tiles >= sms / 2) return 1;
  int splits = (sms + tiles - 1) / tiles;
  if (splits > num_kb / 4) splits = num_kb / 4;
  if (splits < 2) return 1;
  const int kb_per = (num_kb + splits - 1) / splits;
  *kb_per_out = kb_per;
  return (num_kb + kb_per - 1) / kb_per;
}

// Tile-width choice: the widest BN that still yields enough tiles to cover
// the SMs (wide tiles reuse A best; narrow tiles spread a skinny decode GEMM
// over more SMs so the weight stream uses all of HBM).
int choose_bn(int M, int N, int epi) {
  const int sms = num_sms();
  const int num_m = (M + BM - 1) / BM;
  const int cands[4] = {256, 128, 64, 32};
  for (int i = 0; i < 4; ++i) {
    const int bn = cands[i];
    if (N % bn != 0) continue;
    if (epi == kSwiGLU && bn < 64) continue;
    if (num_m * (N / bn) >= sms) return bn;
  }
  for (int i = 3; i >= 0; --i) {
    if (N % cands[i] == 0 && !(epi == kSwiGLU && cands[i] < 64)) return cands[i];
  }
  return 0;
}

void run(const GemmArgs& a, int epi, int bn, cudaStream_t stream, float* ws, int64_t ws_elems) {
  if (a.M <= 0) return;
  if (ws != nullptr && bn == 0 && (a.N % 256) == 0) {
    int kb_per = 0;
    const int splits = plan_splitk(a.M, a.N, a.K, &kb_per);
    if (splits > 1 && (int64_t)splits * a.M * a.N <= ws_elems) {
      if (a.K % 8 != 0) throw std::runtime_error("lunaflux gemm: K must be a multiple of 8");
      launch<256, 4, kSplitF32>(a, stream, splits, kb_per, ws);
      dim3 grid((a.N + 1023) / 1024, a.M);
      if (epi == kSwiGLU) splitk_finalize_kernel<kSwiGLU><<<grid, 256, 0, stream>>>(ws, a.D, a.M, a.N, a.ldd, splits);
      else if (epi == kStoreF32) splitk_finalize_kernel<kStoreF32><<<grid, 256, 0, stream>>>(ws, a.D, a.M, a.N, a.ldd, splits);
      else splitk_finalize_kernel<kStoreBf16><<<grid, 256, 0, stream>>>(ws, a.D, a.M, a.N, a.ldd, splits);
      return;
    }
  }
  if (bn == 0) bn = choose_bn(a.M, a.N, epi);
  if (bn == 0 || a.N % bn != 0) throw std::runtime_error("lunaflux gemm: N must be a multiple of 32");
  if (a.K % 8 != 0) throw std::runtime_error("lunaflux gemm: K must be a multiple of 8");
#define LF_GEMM_CASE(BNV, ST)                                         \
  case BNV:                                                           \
    if (epi == kStoreBf16) launch<BNV, ST, kStoreBf16>(a, stream);    \
    else if (epi == kStoreF32) launch<BNV, ST, kStoreF32>(a, stream); \
    else launch<BNV, ST, kSwiGLU>(a, stream);                         \
    break;
  switch (bn) {
    LF_GEMM_CASE(256, 4)
    LF_GEMM_CASE(128, 6)
    LF_GEMM_CASE(64, 8)
    case 32:
      if (epi == kStoreBf16) launch<32, 8, kStoreBf16>(a, stream);
      else if (epi == kStoreF32) launch<32, 8, kStoreF32>(a, stream);
      else throw std::runtime_error("lunaflux gemm: SwiGLU needs BN >= 64");
      break;
    default:
      throw std::runtime_error("lunaflux gemm: unsupported BN");
  }
#undef LF_GEMM_CASE
}

}  // namespace gemm
}  // namespace lf
