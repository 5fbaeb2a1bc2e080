// Block-scaled fp8 GEMM for sm_100a (tcgen05 kind::f8f6f4, e4m3 x e4m3 -> fp32).
//
//   D[M, N] = sum_kb  sa[m, kb] * sb[n / 128, kb] * (A8[m, kb] . B8[n, kb]^T)
//
// A8: activations, e4m3 [M, K], one fp32 scale per (row, 128-wide K block).
// B8: weights, e4m3 [N, K], one fp32 scale per 128 x 128 block.
// This is the DeepSeek-style block scaling of the 70B fp8 configuration; the
// scales are not MX (ue8m0, 32-wide), so the tensor core cannot apply them.
// Instead every 128-wide K block is accumulated into its own TMEM buffer
// (4 MMAs of K = 32), and the epilogue warps read it back with tcgen05.ld,
// scale it and add it to fp32 register accumulators, while the MMA warp
// already fills the other TMEM buffer with the next K block.
//
// Roles (192 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer (A: 128 x 128 B box, B: 128 x 128 B box, 128-byte swizzle)
//   warp 1      TMEM allocation; lane 0 issues the MMAs
//   warps 2..5  scale-and-accumulate, then the epilogue (bf16 store, fp32
//               store, or SwiGLU over 32-row interleaved gate/up weights)
// All waits are bounded (common.cuh); every TMA load fills only its own CTA.
//
// Split-K (decode shapes with fewer tiles than SMs): a work item is a (tile,
// K range) pair; each item adds its fp32 partial tile into a zeroed fp32
// workspace [M, N] with vector atomics (red.global.add on L2), and a finalize
// kernel applies the epilogue and zeroes the workspace again.  The order of
// the partial sums is not fixed, so split results may differ in the last
// fp32 bits from run to run.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <mutex>
#include <stdexcept>
#include <unordered_map>

#include "common.cuh"
#include "gemm_bf16.h"
#include "gemm_fp8.h"

namespace lf {
namespace fp8 {

constexpr int BM = 128;
constexpr int BN = 128;      // one weight scale block per tile
constexpr int BK = 128;      // 128 e4m3 = 128 bytes = one swizzle row = one scale block
constexpr int STAGES = 6;
constexpr int kThreads = 192;
constexpr int kStageBytes = (BM + BN) * BK;
constexpr int kSmem = STAGES * kStageBytes + 1024 + 256;

enum Epi : int { kBf16 = 0, kF32 = 1, kSwiGLU = 2 };

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const float* __restrict__ sa, int64_t lds_a, const float* __restrict__ sb, void* __restrict__ out,
                    int M, int N, int K, int64_t ldd, int splits, int kb_per, float* __restrict__ ws) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull = empty_bar + STAGES;  // [2] per-K-block TMEM buffers
  uint64_t* tempty = tfull + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = N / BN, tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  const int items = tiles * splits;
  constexpr uint32_t kCols = 2 * BN;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
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
      const uint64_t pol = l2_policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        const int tile = item % tiles, kb0 = (item / tiles) * kb_per;
        const int kb1 = min(num_kb, kb0 + kb_per);
        const int m0 = (tile % num_m) * BM, n0 = (tile / num_m) * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, 31)) { ok = false; break; }
          uint8_t* sa_s = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
          tma_load_2d(sa_s, &tmap_a, &full_bar[stage], kb * BK, m0);
          tma_load_2d_hint(sa_s + BM * BK, &tmap_b, &full_bar[stage], kb * BK, n0, pol);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0, tb = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
        const int kb0 = (item / tiles) * kb_per, kb1 = min(num_kb, kb0 + kb_per);
        for (int kb = kb0; kb < kb1; ++kb, ++tb) {
          const int b = tb & 1;
          if (!mbar_wait(&tempty[b], ((tb >> 1) & 1) ^ 1, 32)) { ok = false; break; }
          if (!mbar_wait(&full_bar[stage], phase, 33)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * kStageBytes);
          const uint32_t b_addr = a_addr + BM * BK;
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            umma_f8_ss(tmem_base + b * BN, sw128_kmajor_desc(a_addr + kk * 32), sw128_kmajor_desc(b_addr + kk * 32),
                       idesc, kk > 0 ? 1u : 0u);
          umma_commit(&empty_bar[stage]);
          umma_commit(&tfull[b]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else {
    const int quad = warp & 3;
    const int ksb = (K + BK - 1) / BK;  // scale blocks per row
    uint32_t tb = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      const int tile = item % tiles, kb0 = (item / tiles) * kb_per;
      const int kb1 = min(num_kb, kb0 + kb_per);
      const int m0 = (tile % num_m) * BM, n0 = (tile / num_m) * BN;
      const int row = m0 + quad * 32 + lane;
      const int rr = row < M ? row : M - 1;
      float acc[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = 0.f;
      const float* sa_row = sa + (size_t)rr * lds_a;
      const float* sb_blk = sb + (size_t)(n0 / 128) * ksb;
      float scale_next = sa_row[kb0] * sb_blk[kb0];
      for (int kb = kb0; kb < kb1; ++kb, ++tb) {
        const int b = tb & 1;
        // this block's scale was loaded during the previous block; the next
        // one is requested before waiting for the accumulator
        const float scale = scale_next;
        if (kb + 1 < kb1) scale_next = sa_row[kb + 1] * sb_blk[kb + 1];
        if (!mbar_wait(&tfull[b], (tb >> 1) & 1, 34)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + b * BN;
        // two halves of 64 columns: four loads in flight per wait
#pragma unroll
        for (int c = 0; c < BN; c += 64) {
          uint32_t r[64];
          tmem_ld_32x32b_x16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(r));
          tmem_ld_32x32b_x16(taddr + c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
          tmem_ld_32x32b_x16(taddr + c + 32, *reinterpret_cast<uint32_t(*)[16]>(r + 32));
          tmem_ld_32x32b_x16(taddr + c + 48, *reinterpret_cast<uint32_t(*)[16]>(r + 48));
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 64; ++j) acc[c + j] = fmaf(__uint_as_float(r[j]), scale, acc[c + j]);
        }
        tc_fence_before();
        mbar_arrive(&tempty[b]);
      }
      if (!ok || row >= M) continue;
      if (splits > 1) {
        float* dst = ws + (size_t)row * N + n0;
#pragma unroll
        for (int j = 0; j < BN; j += 4)
          atomicAdd(reinterpret_cast<float4*>(dst + j), make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]));
        continue;
      }
      if constexpr (EPI == kSwiGLU) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + n0 / 2;
#pragma unroll
        for (int g = 0; g < BN / 64; ++g) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 v;
            uint32_t* p = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c = g * 64 + j + 2 * e;
              p[e] = pack_bf16x2(silu(acc[c]) * acc[c + 32], silu(acc[c + 1]) * acc[c + 33]);
            }
            *reinterpret_cast<uint4*>(dst + g * 32 + j) = v;
          }
        }
      } else if constexpr (EPI == kF32) {
        float* dst = reinterpret_cast<float*>(out) + (size_t)row * ldd + n0;
#pragma unroll
        for (int j = 0; j < BN; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      } else {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + n0;
#pragma unroll
        for (int j = 0; j < BN; j += 8)
          *reinterpret_cast<uint4*>(dst + j) =
              make_uint4(pack_bf16x2(acc[j], acc[j + 1]), pack_bf16x2(acc[j + 2], acc[j + 3]),
                         pack_bf16x2(acc[j + 4], acc[j + 5]), pack_bf16x2(acc[j + 6], acc[j + 7]));
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

// Split-K finalize: out = epilogue(ws), then ws = 0.  One thread per 8
// output columns (bf16 / fp32), or per 8 SwiGLU outputs (16 workspace
// columns: 8 gate, and the 8 up columns 32 further on).
template <int EPI>
__global__ void splitk_finalize_kernel(float* __restrict__ ws, void* __restrict__ out, int M, int N, int64_t ldd) {
  pdl_trigger();
  pdl_wait();
  const int per_row = EPI == kSwiGLU ? N / 16 : N / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * per_row) return;
  const int row = (int)(i / per_row), c = (int)(i % per_row);
  float* src = ws + (size_t)row * N;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  if constexpr (EPI == kSwiGLU) {
    const int g = c / 4, j = (c % 4) * 8;             // group of 64 columns, 8 of its 32 outputs
    float4* gp = reinterpret_cast<float4*>(src + g * 64 + j);
    float4* up = reinterpret_cast<float4*>(src + g * 64 + 32 + j);
    const float4 g0 = gp[0], g1 = gp[1], u0 = up[0], u1 = up[1];
    gp[0] = z; gp[1] = z; up[0] = z; up[1] = z;
    uint4 v = make_uint4(pack_bf16x2(silu(g0.x) * u0.x, silu(g0.y) * u0.y), pack_bf16x2(silu(g0.z) * u0.z, silu(g0.w) * u0.w),
                         pack_bf16x2(silu(g1.x) * u1.x, silu(g1.y) * u1.y), pack_bf16x2(silu(g1.z) * u1.z, silu(g1.w) * u1.w));
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + g * 32 + j) = v;
  } else {
    float4* p = reinterpret_cast<float4*>(src + c * 8);
    const float4 a = p[0], b = p[1];
    p[0] = z;
    p[1] = z;
    if constexpr (EPI == kF32) {
      float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)row * ldd + c * 8);
      d[0] = a;
      d[1] = b;
    } else {
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)row * ldd + c * 8) =
          make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
    }
  }
}

// Per (row, 128-column block) quantisation: scale = amax / 448, q = x / scale.
// One warp per block, 4 elements per lane.
__global__ void act_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M, int K,
                                 __nv_fp8_e4m3* __restrict__ q, float* __restrict__ s, int64_t lds) {
  const int nb = K / 128;
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= M * nb) return;
  const int row = w / nb, blk = w % nb;
  const __nv_bfloat16* src = x + (size_t)row * ldx + blk * 128 + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __bfloat162float(b[i]);
    amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = warp_max(amax);
  const float scale = fmaxf(amax, 1e-12f) / 448.f;
  const float inv = 1.f / scale;
  __nv_fp8x4_e4m3 packed(make_float4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv));
  *reinterpret_cast<__nv_fp8x4_e4m3*>(q + (size_t)row * K + blk * 128 + lane * 4) = packed;
  if (lane == 0) s[(size_t)row * lds + blk] = scale;
}

// ---------------------------------------------------------------------------
namespace {
std::mutex g_mu;
std::unordered_map<uint64_t, CUtensorMap> g_maps;
int sms() {
  static int n = 0;
  if (!n) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
  }
  return n;
}
CUtensorMap map_u8(const void* p, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  const uint64_t key = reinterpret_cast<uint64_t>(p) ^ (rows * 0x9E3779B97F4A7C15ull) ^ (cols << 40) ^ (ld << 20) ^
                       box_rows;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) return it->second;
  if (g_maps.size() > 65536) g_maps.clear();
  CUtensorMap m = gemm::make_tmap_2d(p, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, cols, ld, box_rows, BK,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  g_maps.emplace(key, m);
  return m;
}
template <int EPI>
void launch(const Fp8Args& a, cudaStream_t s, float* ws, int64_t ws_elems) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_fp8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    attr = true;
  }
  const CUtensorMap ta = map_u8(a.A, a.M, a.K, a.lda, BM);
  const CUtensorMap tb = map_u8(a.B, a.N, a.K, a.ldb, BN);
  const int tiles = ((a.M + BM - 1) / BM) * (a.N / BN);
  int kb_per = 0;
  const int splits = (ws != nullptr && (int64_t)a.M * a.N <= ws_elems) ? plan_splits(tiles, a.K / BK, sms(), &kb_per) : 1;
  if (splits == 1) kb_per = a.K / BK;
  const int items = tiles * splits;
  const int grid = items < sms() ? items : sms();
  gemm_fp8_kernel<EPI><<<grid, kThreads, kSmem, s>>>(ta, tb, a.sa, a.lds_a, a.sb, a.D, a.M, a.N, a.K, a.ldd, splits,
                                                     kb_per, ws);
  if (splits > 1) {
    const int64_t threads = (int64_t)a.M * (EPI == kSwiGLU ? a.N / 16 : a.N / 8);
    launch_k(splitk_finalize_kernel<EPI>, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, s, 1, ws, a.D, a.M, a.N,
             a.ldd);
  }
}
}  // namespace

int plan_splits(int tiles, int num_kb, int sms, int* kb_per) {
  // Fill about one wave: as many K splits as the tiles leave SMs free, each
  // split at least 4 K blocks (512 channels) so the pipeline fill amortises.
  // Only where the tiles leave more than half the SMs idle and K is long
  // (>= 32 blocks): measured on the 70B TP 8 shapes at 128 rows, splitting
  // qkv (10 tiles, K 8192) took 33.8 -> 15.4 us and gate/up (56 tiles)
  // 35.9 -> 29.7 us, while o (64 tiles, K 1024) went 13.3 -> 19.4 us and
  // down (K 3584) 20.5 -> 23.6 us: there the fp32 partial traffic and the
  // finalize pass cost more than the idle SMs return.
  if (tiles * 2 > sms || num_kb < 32) {
    *kb_per = num_kb;
    return 1;
  }
  int splits = sms / tiles;
  const int max_splits = num_kb / 4;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  const int per = (num_kb + splits - 1) / splits;
  *kb_per = per;
  return (num_kb + per - 1) / per;
}

void run(const Fp8Args& a, int epi, cudaStream_t s, float* ws, int64_t ws_elems) {
  if (a.M <= 0) return;
  if (a.N % BN != 0 || a.K % BK != 0) throw std::runtime_error("lunaflux fp8 gemm: N and K must be multiples of 128");
  if (epi == kSwiGLU) launch<kSwiGLU>(a, s, ws, ws_elems);
  else if (epi == kF32) launch<kF32>(a, s, ws, ws_elems);
  else launch<kBf16>(a, s, ws, ws_elems);
}

void act_quant(const void* x, int64_t ldx, int M, int K, void* q, float* s, int64_t lds, cudaStream_t st) {
  if (M <= 0) return;
  if (K % 128 != 0) throw std::runtime_error("lunaflux act_quant: K must be a multiple of 128");
  const int warps = M * (K / 128);
  act_quant_kernel<<<(warps * 32 + 255) / 256, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, K,
                                                              reinterpret_cast<__nv_fp8_e4m3*>(q), s, lds);
}

}  // namespace fp8
}  // namespace lf
