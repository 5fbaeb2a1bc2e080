// Allocation-free entry point of the tcgen05 bf16 GEMM; see gemm_noalloc.h for
// who needs it, the scratch contract and the set-up rule.
//
// Its plan is not the allocating entry point's.  lf::gemm::run sends skinny
// shapes to cluster split-K (partial tiles summed through distributed shared
// memory, no global scratch) and 129..256-row shapes to 256-row tiles.  This
// entry point keeps the slab split-K design instead: each K slice writes an
// fp32 [M, N] slab into the file-scope scratch array below and a finalize
// kernel sums the slabs in split order and applies the epilogue.  Other shapes
// use the persistent kernel with the tile width of choose_bn.  The summation
// order therefore differs from run(): results agree within bf16 rounding, not
// bitwise.  Both the split plan and the tile width are computed for the SM
// count of the current device.  TMA descriptors are encoded on the stack (no
// descriptor cache); nothing is allocated on the device or the host.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "gemm_bf16.h"
#include "gemm_bf16_kernel.cuh"
#include "gemm_noalloc.h"

static __device__ __align__(256) float lf_gemm_noalloc_scratch[LF_GEMM_NOALLOC_SCRATCH_FLOATS];

namespace lf {
namespace gemm {
namespace {

constexpr int kMaxDevices = 64;

struct DeviceSetup {
  bool done = false;
  bool ok = false;
  float* scratch = nullptr;  // device address of lf_gemm_noalloc_scratch on this device
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

template <int BN, int STAGES, int EPI>
cudaError_t set_smem_attr() {
  return cudaFuncSetAttribute(gemm_bf16_kernel<BN, STAGES, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Smem<BN, STAGES>::kTotal);
}

// Once per device, with that device current: resolve the scratch address and
// raise the dynamic shared-memory limit of every kernel this file launches.
// A failed set-up is not remembered: the next call on the device tries again.
bool setup_device(int dev) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  DeviceSetup& s = g_setup[dev];
  if (s.done) return s.ok;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, lf_gemm_noalloc_scratch) != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return false;
  }
  s.scratch = static_cast<float*>(p);
  cudaError_t e = cudaSuccess;
  const cudaError_t errs[] = {
      set_smem_attr<256, 4, kStoreBf16>(), set_smem_attr<256, 4, kStoreF32>(), set_smem_attr<256, 4, kSwiGLU>(),
      set_smem_attr<256, 4, kSplitF32>(),  set_smem_attr<128, 6, kStoreBf16>(), set_smem_attr<128, 6, kStoreF32>(),
      set_smem_attr<128, 6, kSwiGLU>(),    set_smem_attr<64, 8, kStoreBf16>(),  set_smem_attr<64, 8, kStoreF32>(),
      set_smem_attr<64, 8, kSwiGLU>(),     set_smem_attr<32, 8, kStoreBf16>(),  set_smem_attr<32, 8, kStoreF32>()};
  for (cudaError_t x : errs)
    if (x != cudaSuccess) e = x;
  if (e != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  s.done = true;
  return s.ok = true;
}

int sm_count(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Launches with cudaLaunchKernelEx so that each launch reports its own error
// (the caller's earlier, unrelated errors are neither read nor cleared).
template <typename... Params, typename... Args>
cudaError_t launch_ex(void (*kfn)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  return cudaLaunchKernelEx(&cfg, kfn, static_cast<Params>(args)...);
}

template <int BN, int STAGES, int EPI>
cudaError_t launch_stack(const GemmArgs& a, cudaStream_t stream, int sms, int splits, int kb_per, float* ws) {
  // Tensor maps are built on the stack: no descriptor cache, no allocation.
  const CUtensorMap ta = make_tmap_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.lda, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tb = make_tmap_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, a.ldb, BN, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const int units = ((a.M + BM - 1) / BM) * (a.N / BN) * splits;
  const int grid = units < sms ? units : sms;
  if (kb_per <= 0) kb_per = (a.K + BK - 1) / BK;
  void* out = (EPI == kSplitF32) ? static_cast<void*>(ws) : a.D;
  const int ldd = (EPI == kSplitF32) ? a.N : (int)a.ldd;
  return launch_ex(gemm_bf16_kernel<BN, STAGES, EPI>, dim3(grid), dim3(kThreads), Smem<BN, STAGES>::kTotal, stream,
                   ta, tb, out, a.M, a.N, a.K, ldd, splits, kb_per, ArArgs{}, (const int*)nullptr, 0, RopeArgs{});
}

template <int EPI>
cudaError_t launch_bn(const GemmArgs& a, int bn, cudaStream_t stream, int sms) {
  switch (bn) {
    case 256: return launch_stack<256, 4, EPI>(a, stream, sms, 1, 0, nullptr);
    case 128: return launch_stack<128, 6, EPI>(a, stream, sms, 1, 0, nullptr);
    case 64: return launch_stack<64, 8, EPI>(a, stream, sms, 1, 0, nullptr);
    default:
      if constexpr (EPI != kSwiGLU) return launch_stack<32, 8, EPI>(a, stream, sms, 1, 0, nullptr);
      return cudaErrorInvalidValue;
  }
}

}  // namespace
}  // namespace gemm
}  // namespace lf

extern "C" int lf_gemm_bf16_noalloc(const void* A, const void* B, void* D, int M, int N, int K, int64_t lda,
                                    int64_t ldb, int64_t ldd, int epi, void* stream_ptr) {
  using namespace lf::gemm;
  if (A == nullptr || B == nullptr || D == nullptr || M <= 0 || N <= 0 || K <= 0) return LF_NOALLOC_BAD_ARGUMENT;
  if (epi < kStoreBf16 || epi > kSwiGLU) return LF_NOALLOC_BAD_ARGUMENT;
  if (N % 32 != 0 || K % 8 != 0 || (epi == kSwiGLU && N % 64 != 0)) return LF_NOALLOC_BAD_ARGUMENT;
  if (lda < K || ldb < K || (lda % 8) != 0 || (ldb % 8) != 0) return LF_NOALLOC_BAD_ARGUMENT;
  if (ldd < (epi == kSwiGLU ? N / 2 : N) || (ldd % 8) != 0) return LF_NOALLOC_BAD_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(D)) & 15)
    return LF_NOALLOC_BAD_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return LF_NOALLOC_SETUP_FAILED;
  if (!setup_device(dev)) return LF_NOALLOC_SETUP_FAILED;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const GemmArgs a{A, B, D, M, N, K, lda, ldb, ldd};
  const int sms = sm_count(dev);
  cudaError_t err = cudaSuccess;
  try {
    // Slab split-K for skinny shapes (scratch in use), else persistent tiles.
    int kb_per = 0;
    const int splits = (N % 256 == 0) ? plan_splitk_sms(M, N, K, sms, &kb_per) : 1;
    if (splits > 1) {
      if ((uint64_t)splits * M * N > LF_GEMM_NOALLOC_SCRATCH_FLOATS) return LF_NOALLOC_TOO_LARGE;
      float* ws = g_setup[dev].scratch;
      err = launch_stack<256, 4, kSplitF32>(a, stream, sms, splits, kb_per, ws);
      if (err == cudaSuccess) {
        const dim3 grid((N + 1023) / 1024, M);
        const float* cws = ws;
        if (epi == kSwiGLU)
          err = launch_ex(splitk_finalize_kernel<kSwiGLU>, grid, dim3(256), 0, stream, cws, D, M, N, ldd, splits);
        else if (epi == kStoreF32)
          err = launch_ex(splitk_finalize_kernel<kStoreF32>, grid, dim3(256), 0, stream, cws, D, M, N, ldd, splits);
        else
          err = launch_ex(splitk_finalize_kernel<kStoreBf16>, grid, dim3(256), 0, stream, cws, D, M, N, ldd, splits);
      }
    } else {
      const int bn = choose_bn_sms(M, N, epi, sms);
      if (bn == 0) return LF_NOALLOC_BAD_ARGUMENT;
      if (epi == kSwiGLU) err = launch_bn<kSwiGLU>(a, bn, stream, sms);
      else if (epi == kStoreF32) err = launch_bn<kStoreF32>(a, bn, stream, sms);
      else err = launch_bn<kStoreBf16>(a, bn, stream, sms);
    }
  } catch (...) {
    return LF_NOALLOC_BAD_ARGUMENT;  // tensor-map encoding rejected the operands
  }
  return err == cudaSuccess ? LF_NOALLOC_OK : LF_NOALLOC_LAUNCH_FAILED;
}
