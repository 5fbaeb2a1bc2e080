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
// Shape variants chosen by run():
//   * skinny GEMMs (the tiles would leave more than half of the SMs idle):
//     cluster split-K, gemm_cluster_splitk_kernel (one cluster of up to 8
//     CTAs per tile, partials summed through distributed shared memory);
//   * 129..256 rows: 256-row tiles (two M=128 MMAs per weight slab);
//   * otherwise the widest BN that still covers the SMs.
// The fused all-reduce epilogue (kAllReduceBf16), the fp32 split slabs
// (kSplitF32) and the grouped mixture-of-experts mode share the kernel.
//
// All waits are bounded (common.cuh); every TMA load fills only its own CTA.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "gemm_bf16.h"

#include "gemm_bf16_kernel.cuh"

namespace lf {
namespace gemm {

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

template <int BN, int STAGES, int EPI, int MB = 1>
static void launch(const GemmArgs& a, cudaStream_t stream, int splits = 1, int kb_per = 0, float* ws = nullptr,
                   const ArArgs& ar = ArArgs{}, const RopeArgs& rope = RopeArgs{}) {
  using S = Smem<BN, STAGES, MB>;
  auto kfn = gemm_bf16_kernel<BN, STAGES, EPI, MB>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    attr_set = true;
  }
  CUtensorMap ta = cached_tmap_bf16(a.A, a.M, a.K, a.lda, BM);
  CUtensorMap tb = cached_tmap_bf16(a.B, a.N, a.K, a.ldb, BN);
  const int tiles = ((a.M + MB * BM - 1) / (MB * BM)) * (a.N / BN) * splits;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  if (kb_per <= 0) kb_per = (a.K + BK - 1) / BK;
  const int* no_groups = nullptr;
  if (EPI == kSplitF32) {
    launch_k(kfn, dim3(grid), dim3(kThreads), S::kTotal, stream, 1, ta, tb, static_cast<void*>(ws), a.M, a.N, a.K, a.N,
             splits, kb_per, ArArgs{}, no_groups, 0, RopeArgs{});
  } else {
    launch_k(kfn, dim3(grid), dim3(threads_for(EPI)), S::kTotal, stream, 1, ta, tb, a.D, a.M, a.N, a.K, (int)a.ldd,
             splits, kb_per, ar, no_groups, 0, rope);
  }
}

// Split-K plan for skinny GEMMs: 256-wide tiles (so the activations are
// re-read from L2 as few times as possible) and enough K-splits to cover the
// SMs, each split at least 4 k-blocks.  Returns splits (1 = no split).
int plan_splitk(int M, int N, int K, int* kb_per_out) { return plan_splitk_sms(M, N, K, num_sms(), kb_per_out); }

int plan_splitk_sms(int M, int N, int K, int sms, int* kb_per_out) {
  const int num_m = (M + BM - 1) / BM;
  const int num_kb = (K + BK - 1) / BK;
  if (N % 256 != 0) return 1;
  const int tiles = num_m * (N / 256);
  if (tiles >= sms / 2) return 1;
  // one wave: tiles * splits <= SMs (a partial second wave doubles the time)
  int splits = sms / tiles;
  if (splits > num_kb / 4) splits = num_kb / 4;
  if (splits < 2) return 1;
  const int kb_per = (num_kb + splits - 1) / splits;
  *kb_per_out = kb_per;
  return (num_kb + kb_per - 1) / kb_per;
}

// Cluster split-K (skinny decode GEMMs): one cluster of c CTAs per output
// tile, the partial tiles summed through distributed shared memory.
template <int BN, int STAGES, int OUT, int MB = 1>
static bool cluster_fits(int c, int clusters) {
  using S = Smem<BN, STAGES, MB>;
  static int cached[9] = {0};
  if (cached[c] == 0) {
    auto kfn = gemm_cluster_splitk_kernel<BN, STAGES, OUT, MB>;
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c * clusters, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::kTotal;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = -1;
    }
    cached[c] = n;
  }
  return cached[c] >= clusters;
}

template <int BN, int STAGES, int OUT, int MB = 1>
static void launch_cluster(const GemmArgs& a, int c, int kb_per, void* out, int64_t ldd, cudaStream_t stream,
                           const ar::LLArgs& ll = ar::LLArgs{}, const RopeArgs& rope = RopeArgs{}) {
  using S = Smem<BN, STAGES, MB>;
  auto kfn = gemm_cluster_splitk_kernel<BN, STAGES, OUT, MB>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    attr_set = true;
  }
  CUtensorMap ta = cached_tmap_bf16(a.A, a.M, a.K, a.lda, BM);
  CUtensorMap tb = cached_tmap_bf16(a.B, a.N, a.K, a.ldb, BN);
  const int tiles = ((a.M + MB * BM - 1) / (MB * BM)) * (a.N / BN);
  launch_k(kfn, dim3(tiles * c), dim3(kThreads), S::kTotal, stream, (unsigned)c, ta, tb, out, a.M, a.N, a.K, (int)ldd,
           kb_per, ll, rope);
}

// 256-row cluster tiles (MB = 2) for 129..256-row GEMMs: off unless enabled
// (LUNAFLUX_GEMM_CLUSTER_MB2=1 or set_cluster_mb2).  Measured slower than
// 128-row tiles on the Llama-3-8B decode shapes (fewer CTAs in flight, two
// reductions in turn), so the default plan does not use them.
static int g_cluster_mb2 = -1;

void set_cluster_mb2(int on) { g_cluster_mb2 = on ? 1 : 0; }

static bool cluster_mb2_enabled() {
  if (g_cluster_mb2 < 0) {
    const char* e = getenv("LUNAFLUX_GEMM_CLUSTER_MB2");
    g_cluster_mb2 = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return g_cluster_mb2 == 1;
}

// 256-row variant: tiles of 256 x 256, so each weight slab is staged once for
// both M-blocks.  Returns the cluster size (0: not applicable).
static int plan_cluster_mb2(int M, int N, int K, int epi, int* kb_per_out) {
  const int sms = num_sms();
  const int num_kb = (K + BK - 1) / BK;
  if (M <= BM || M > 2 * BM || N % 256 != 0 || K % 8 != 0) return 0;
  const int tiles = N / 256;
  if (tiles >= sms / 2) return 0;
  int c = sms / tiles;
  if (c > 8) c = 8;
  if (c > num_kb / 2) c = num_kb / 2;
  for (; c >= 2; --c) {
    const bool fits = epi == kSwiGLU ? cluster_fits<256, 3, kSwiGLU, 2>(c, tiles)
                      : epi == kStoreF32 ? cluster_fits<256, 3, kStoreF32, 2>(c, tiles)
                                         : cluster_fits<256, 3, kStoreBf16, 2>(c, tiles);
    if (fits) break;
  }
  if (c < 2) return 0;
  const int kb_per = (num_kb + c - 1) / c;
  c = (num_kb + kb_per - 1) / kb_per;  // no empty slice
  if (c < 2) return 0;
  *kb_per_out = kb_per;
  return c;
}

// Plan: BN 256 when the 256-wide tiles times up to 8 splits reach half of
// the SMs, else BN 128; as many splits (cluster size, <= 8) as one wave allows, with
// at least two k-blocks per split; only when the plain tiles would leave more
// than half of the SMs idle.  Returns the cluster size (0: no split).
int plan_cluster(int M, int N, int K, int epi, int* bn_out, int* kb_per_out, int* mb_out) {
  const int sms = num_sms();
  const int num_m = (M + BM - 1) / BM;
  const int num_kb = (K + BK - 1) / BK;
  if (mb_out != nullptr) *mb_out = 1;
  if (N % 128 != 0 || K % 8 != 0) return 0;
  if (cluster_mb2_enabled()) {
    const int c2 = plan_cluster_mb2(M, N, K, epi, kb_per_out);
    if (c2 >= 2) {
      *bn_out = 256;
      if (mb_out != nullptr) *mb_out = 2;
      return c2;
    }
  }
  const int t256 = N % 256 == 0 ? num_m * (N / 256) : 0;
  const int t128 = num_m * (N / 128);
  if ((t256 ? t256 : t128) >= sms / 2) return 0;
  // 256-wide tiles halve the activation bytes staged per weight byte; narrower
  // tiles only when the 256-wide ones cannot reach half of the SMs
  const int bn = (t256 && t256 * 8 >= sms / 2) ? 256 : 128;
  const int tiles = bn == 256 ? t256 : t128;
  int c = sms / tiles;
  if (c > 8) c = 8;
  if (c > num_kb / 2) c = num_kb / 2;
  for (; c >= 2; --c) {
    bool fits;
    if (bn == 256) {
      fits = epi == kSwiGLU ? cluster_fits<256, 4, kSwiGLU>(c, tiles)
             : epi == kStoreF32 ? cluster_fits<256, 4, kStoreF32>(c, tiles)
                                : cluster_fits<256, 4, kStoreBf16>(c, tiles);
    } else {
      fits = epi == kSwiGLU ? cluster_fits<128, 6, kSwiGLU>(c, tiles)
             : epi == kStoreF32 ? cluster_fits<128, 6, kStoreF32>(c, tiles)
                                : cluster_fits<128, 6, kStoreBf16>(c, tiles);
    }
    if (fits) break;
  }
  if (c < 2) return 0;
  const int kb_per = (num_kb + c - 1) / c;
  c = (num_kb + kb_per - 1) / kb_per;  // no empty slice
  if (c < 2) return 0;
  *bn_out = bn;
  *kb_per_out = kb_per;
  return c;
}

static bool run_cluster(const GemmArgs& a, int epi, void* out, int64_t ldd, cudaStream_t stream) {
  int bn = 0, kb_per = 0, mb = 1;
  const int c = plan_cluster(a.M, a.N, a.K, epi, &bn, &kb_per, &mb);
  if (c < 2) return false;
  if (mb == 2) {
    if (epi == kSwiGLU) launch_cluster<256, 3, kSwiGLU, 2>(a, c, kb_per, out, ldd, stream);
    else if (epi == kStoreF32) launch_cluster<256, 3, kStoreF32, 2>(a, c, kb_per, out, ldd, stream);
    else launch_cluster<256, 3, kStoreBf16, 2>(a, c, kb_per, out, ldd, stream);
  } else if (bn == 256) {
    if (epi == kSwiGLU) launch_cluster<256, 4, kSwiGLU>(a, c, kb_per, out, ldd, stream);
    else if (epi == kStoreF32) launch_cluster<256, 4, kStoreF32>(a, c, kb_per, out, ldd, stream);
    else launch_cluster<256, 4, kStoreBf16>(a, c, kb_per, out, ldd, stream);
  } else {
    if (epi == kSwiGLU) launch_cluster<128, 6, kSwiGLU>(a, c, kb_per, out, ldd, stream);
    else if (epi == kStoreF32) launch_cluster<128, 6, kStoreF32>(a, c, kb_per, out, ldd, stream);
    else launch_cluster<128, 6, kStoreBf16>(a, c, kb_per, out, ldd, stream);
  }
  return true;
}

}  // namespace gemm
}  // namespace lf

#include "gemm_bf16_2sm.cuh"

namespace lf {
namespace gemm {

// Tile-width choice: the widest BN that still yields enough tiles to cover
// the SMs (wide tiles reuse A best; narrow tiles spread a skinny decode GEMM
// over more SMs so the weight stream uses all of HBM).
int choose_bn(int M, int N, int epi) { return choose_bn_sms(M, N, epi, num_sms()); }

int choose_bn_sms(int M, int N, int epi, int sms) {
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
  (void)ws;
  (void)ws_elems;
  if (bn == 0 && run_pair(a, epi, stream)) return;  // CTA-pair kernel for large GEMMs (LUNAFLUX_GEMM_2SM=0: off)
  if (bn == 0 && run_cluster(a, epi, a.D, a.ldd, stream)) return;
  if (bn == 0 && a.M > BM && a.M <= 2 * BM && a.N % 256 == 0 && a.K % 8 == 0) {
    // 129..256 rows (decode batches): 256-row tiles, each weight slab staged
    // once for both M-blocks
    if (epi == kStoreBf16) launch<256, 3, kStoreBf16, 2>(a, stream);
    else if (epi == kStoreF32) launch<256, 3, kStoreF32, 2>(a, stream);
    else launch<256, 3, kSwiGLU, 2>(a, stream);
    return;
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

// GEMM + tensor-parallel all-reduce in one kernel: D = sum over ranks of
// A_r . B_r^T (row-parallel projections).  Skinny shapes use split-K with the
// all-reduce fused into the persistent finalize kernel instead.
static int finalize_ar_grid(int64_t vecs) {
  // Every CTA must be resident (the kernel has a grid-wide barrier), and the
  // grid must be the same on every rank (a function of the shape, the kernel
  // and the device only).
  static int per_sm = 0;
  if (per_sm == 0) {
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, splitk_finalize_ar_kernel, 256, 0);
    if (per_sm < 1) throw std::runtime_error("lunaflux partials_allreduce: kernel cannot be resident");
    if (per_sm > 2) per_sm = 2;
  }
  const int64_t cap = (int64_t)per_sm * num_sms();
  const int64_t want = (vecs + 255) / 256;
  return (int)(want < cap ? (want < 1 ? 1 : want) : cap);
}

void run_allreduce(const GemmArgs& a, const ArArgs& ar, cudaStream_t stream, float* ws, int64_t ws_elems) {
  if (a.M <= 0) return;
  if (ar.world < 1 || ar.world > kMaxRanks || ar.rank < 0 || ar.rank >= ar.world)
    throw std::runtime_error("lunaflux gemm_allreduce: bad rank or world size");
  if (a.N % 32 != 0 || a.K % 8 != 0) throw std::runtime_error("lunaflux gemm_allreduce: N % 32 and K % 8 required");
  int kb_per = 0;
  const int splits = (ws != nullptr && a.N % 256 == 0) ? plan_splitk(a.M, a.N, a.K, &kb_per) : 1;
  if (splits > 1 && (int64_t)splits * a.M * a.N <= ws_elems) {
    launch<256, 4, kSplitF32>(a, stream, splits, kb_per, ws);
    partials_allreduce(ws, a.M, a.N, splits, ar, stream);
    return;
  }
  const int bn = choose_bn(a.M, a.N, kStoreBf16);
  const int tiles = ((a.M + BM - 1) / BM) * (a.N / bn);
  if (tiles > ar.cnt_capacity - kFinReserved) throw std::runtime_error("lunaflux gemm_allreduce: too many tiles for the counters");
  switch (bn) {
    case 256: launch<256, 4, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
    case 128: launch<128, 6, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
    case 64: launch<64, 8, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
    default: launch<32, 8, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
  }
}

void run_reduce_scatter(const GemmArgs& a, const ArArgs& ar, cudaStream_t stream) {
  if (a.M <= 0) return;
  if (ar.world < 1 || ar.world > kMaxRanks || ar.rank < 0 || ar.rank >= ar.world)
    throw std::runtime_error("lunaflux gemm_reduce_scatter: bad rank or world size");
  if (ar.rs_rows <= 0 || ar.rs_rows % BM != 0 || (int64_t)ar.rs_rows * ar.world != a.M || ar.rs_out == nullptr)
    throw std::runtime_error("lunaflux gemm_reduce_scatter: M must be world * rows, rows a multiple of 128");
  if (a.N % 32 != 0 || a.K % 8 != 0) throw std::runtime_error("lunaflux gemm_reduce_scatter: N % 32 and K % 8 required");
  const int bn = choose_bn(a.M, a.N, kStoreBf16);
  const int tiles = (a.M / BM) * (a.N / bn);
  if (tiles > ar.cnt_capacity - kFinReserved)
    throw std::runtime_error("lunaflux gemm_reduce_scatter: too many tiles for the counters");
  switch (bn) {
    case 256: launch<256, 4, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
    case 128: launch<128, 6, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
    case 64: launch<64, 8, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
    default: launch<32, 8, kAllReduceBf16>(a, stream, 1, 0, nullptr, ar); break;
  }
}

// One kernel for the decode projection and its all-reduce (the cluster
// split-K GEMM whose epilogue runs the low-latency protocol): off unless
// LUNAFLUX_FUSED_LL_GEMM=1 or set_ll_gemm_fused(1).
static int g_ll_gemm_fused = -1;

void set_ll_gemm_fused(int on) { g_ll_gemm_fused = on ? 1 : 0; }

static bool ll_gemm_fused_enabled() {
  if (g_ll_gemm_fused < 0) {
    const char* e = getenv("LUNAFLUX_FUSED_LL_GEMM");
    g_ll_gemm_fused = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return g_ll_gemm_fused == 1;
}

void run_allreduce_ll(const GemmArgs& a, const ar::LLArgs& ll, cudaStream_t stream, float* ws, int64_t ws_elems) {
  if (a.M <= 0) return;
  if (a.N % 256 != 0 || a.K % 8 != 0) throw std::runtime_error("lunaflux gemm_allreduce_ll: N % 256 and K % 8 required");
  if (ll.world < 1 || ll.world > ar::kMaxRanks || ll.rank < 0 || ll.rank >= ll.world)
    throw std::runtime_error("lunaflux gemm_allreduce_ll: rank");
  if (ll_gemm_fused_enabled() && (int64_t)a.M * a.N / 2 <= ll.max_pairs) {
    int bn = 0, kb_per = 0, mb = 1;
    const int c = plan_cluster(a.M, a.N, a.K, kStoreF32, &bn, &kb_per, &mb);
    if (c >= 2 && mb == 1) {
      // every CTA of the grid is resident at once (the plan keeps the grid
      // within one wave), as the cross-rank waits of the epilogue require
      if (bn == 256) launch_cluster<256, 4, kAllReduceLL>(a, c, kb_per, a.D, a.ldd, stream, ll);
      else launch_cluster<128, 6, kAllReduceLL>(a, c, kb_per, a.D, a.ldd, stream, ll);
      return;
    }
  }
  if ((int64_t)a.M * a.N > ws_elems) throw std::runtime_error("lunaflux gemm_allreduce_ll: workspace too small");
  // this rank's fp32 partial [M, N] in ws (cluster split-K when it pays), then the all-reduce
  run(GemmArgs{a.A, a.B, ws, a.M, a.N, a.K, a.lda, a.ldb, a.N}, kStoreF32, 0, stream);
  ar::finalize_ll(ws, 1, a.M, a.N, reinterpret_cast<__nv_bfloat16*>(a.D), a.ldd, ll, stream);
}

bool run_qkv_rope(const GemmArgs& a, const RopeArgs& rope, cudaStream_t stream) {
  if (a.M <= 0) return true;
  if (a.N != (rope.Hq + 2 * rope.Hkv) * 128 || a.K % 8 != 0) return false;
  if (run_pair(a, kQkvRope, stream, rope)) return true;   // large (prefill) shapes on CTA pairs
  int bn = 0, kb_per = 0, mb = 1;
  const int c = plan_cluster(a.M, a.N, a.K, kStoreBf16, &bn, &kb_per, &mb);
  if (c >= 2 && mb == 1) {
    if (bn == 256) launch_cluster<256, 4, kQkvRope>(a, c, kb_per, a.D, a.ldd, stream, ar::LLArgs{}, rope);
    else launch_cluster<128, 6, kQkvRope>(a, c, kb_per, a.D, a.ldd, stream, ar::LLArgs{}, rope);
    return true;
  }
  if (c < 2 && a.M > BM && a.M <= 2 * BM && a.N % 256 == 0) {
    launch<256, 3, kQkvRope, 2>(a, stream, 1, 0, nullptr, ArArgs{}, rope);
    return true;
  }
  if (c >= 2) return false;  // a 256-row cluster plan: no fused variant
  const int b = choose_bn(a.M, a.N, kStoreBf16);
  if (b == 256) launch<256, 4, kQkvRope>(a, stream, 1, 0, nullptr, ArArgs{}, rope);
  else if (b == 128) launch<128, 6, kQkvRope>(a, stream, 1, 0, nullptr, ArArgs{}, rope);
  else return false;
  return true;
}

// Grouped GEMM (mixture-of-experts): A [M_max, K] rows in expert segments
// groups[0..num_groups] (device memory, multiples of BM), B [num_groups * N, K]
// the experts' stacked weights, D [M_max, N] (or [M_max, N / 2] for SwiGLU).
template <int BN, int STAGES, int EPI>
static void launch_grouped(const GemmArgs& a, const int* groups, int num_groups, cudaStream_t stream) {
  using S = Smem<BN, STAGES>;
  auto kfn = gemm_bf16_kernel<BN, STAGES, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    attr_set = true;
  }
  CUtensorMap ta = cached_tmap_bf16(a.A, a.M, a.K, a.lda, BM);
  CUtensorMap tb = cached_tmap_bf16(a.B, (uint64_t)a.N * num_groups, a.K, a.ldb, BN);
  const int tiles = ((a.M + BM - 1) / BM) * (a.N / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kfn<<<grid, kThreads, S::kTotal, stream>>>(ta, tb, a.D, a.M, a.N, a.K, a.ldd, 1, (a.K + BK - 1) / BK, ArArgs{},
                                             groups, num_groups, RopeArgs{});
}

void partials_allreduce(const float* ws, int M, int N, int splits, const ArArgs& ar, cudaStream_t stream) {
  if (M <= 0) return;
  if (N % 8 != 0) throw std::runtime_error("lunaflux partials_allreduce: N % 8 required");
  if (ar.cnt_capacity < 64) throw std::runtime_error("lunaflux partials_allreduce: counter capacity");
  const int grid = finalize_ar_grid((int64_t)M * N / 8);
  splitk_finalize_ar_kernel<<<grid, 256, 0, stream>>>(ws, M, N, splits, ar);
}

void run_grouped(const GemmArgs& a, const int* groups, int num_groups, int epi, cudaStream_t stream, int align) {
  if (a.M <= 0) return;
  // segments of whole 256-row tiles: the CTA-pair kernel, one expert per tile
  if (align == 256 && a.M % 256 == 0 && (epi == kStoreBf16 || epi == kSwiGLU) &&
      run_pair(a, epi, stream, RopeArgs{}, groups, num_groups))
    return;
  if (a.M % BM != 0) throw std::runtime_error("lunaflux grouped gemm: M_max must be a multiple of 128");
  if (a.K % 8 != 0 || a.N % 64 != 0) throw std::runtime_error("lunaflux grouped gemm: K % 8 and N % 64 required");
  const int bn = a.N % 256 == 0 && ((a.M / BM) * (a.N / 256) >= num_sms()) ? 256 : (a.N % 128 == 0 ? 128 : 64);
  if (epi == kSwiGLU) {
    if (bn == 256) launch_grouped<256, 4, kSwiGLU>(a, groups, num_groups, stream);
    else if (bn == 128) launch_grouped<128, 6, kSwiGLU>(a, groups, num_groups, stream);
    else launch_grouped<64, 8, kSwiGLU>(a, groups, num_groups, stream);
  } else {
    if (bn == 256) launch_grouped<256, 4, kStoreBf16>(a, groups, num_groups, stream);
    else if (bn == 128) launch_grouped<128, 6, kStoreBf16>(a, groups, num_groups, stream);
    else launch_grouped<64, 8, kStoreBf16>(a, groups, num_groups, stream);
  }
}

}  // namespace gemm
}  // namespace lf
