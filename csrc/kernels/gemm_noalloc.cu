// Allocation-free entry point of the tcgen05 bf16 GEMM; see gemm_noalloc.h for
// who needs it, the scratch contract and the set-up rule.
//
// It plans the launch exactly as the allocating entry point (lf::gemm::run
// with a workspace) does: the same tile width and the same split-K plan, the
// same kernels.  The differences: the split-K slabs live in the file-scope
// array below instead of a caller workspace, the TMA descriptors are encoded
// on the stack (no descriptor cache), and nothing is allocated on the device
// or the host.
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
bool setup_device(int dev) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  DeviceSetup& s = g_setup[dev];
  if (s.done) return s.ok;
  s.done = true;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, lf_gemm_noalloc_scratch) != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return s.ok = false;
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
    return s.ok = false;
  }
  return s.ok = true;
}

int sm_count(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

template <int BN, int STAGES, int EPI>
void launch_stack(const GemmArgs& a, cudaStream_t stream, int sms, int splits, int kb_per, float* ws) {
  // Tensor maps are built on the stack: no descriptor cache, no allocation.
  const CUtensorMap ta = make_tmap_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.lda, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tb = make_tmap_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, a.ldb, BN, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const int units = ((a.M + BM - 1) / BM) * (a.N / BN) * splits;
  const int grid = units < sms ? units : sms;
  if (kb_per <= 0) kb_per = (a.K + BK - 1) / BK;
  if (EPI == kSplitF32) {
    gemm_bf16_kernel<BN, STAGES, EPI><<<grid, kThreads, Smem<BN, STAGES>::kTotal, stream>>>(
        ta, tb, ws, a.M, a.N, a.K, a.N, splits, kb_per, ArArgs{}, nullptr, 0, RopeArgs{});
  } else {
    gemm_bf16_kernel<BN, STAGES, EPI><<<grid, kThreads, Smem<BN, STAGES>::kTotal, stream>>>(
        ta, tb, a.D, a.M, a.N, a.K, (int)a.ldd, splits, kb_per, ArArgs{}, nullptr, 0, RopeArgs{});
  }
}

template <int EPI>
void launch_bn(const GemmArgs& a, int bn, cudaStream_t stream, int sms) {
  switch (bn) {
    case 256: launch_stack<256, 4, EPI>(a, stream, sms, 1, 0, nullptr); break;
    case 128: launch_stack<128, 6, EPI>(a, stream, sms, 1, 0, nullptr); break;
    case 64: launch_stack<64, 8, EPI>(a, stream, sms, 1, 0, nullptr); break;
    default:
      if constexpr (EPI != kSwiGLU) launch_stack<32, 8, EPI>(a, stream, sms, 1, 0, nullptr);
      break;
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
  try {
    // The same plan as the allocating path: split K for skinny shapes.
    int kb_per = 0;
    const int splits = (N % 256 == 0) ? plan_splitk(M, N, K, &kb_per) : 1;
    if (splits > 1) {
      if ((uint64_t)splits * M * N > LF_GEMM_NOALLOC_SCRATCH_FLOATS) return LF_NOALLOC_TOO_LARGE;
      float* ws = g_setup[dev].scratch;
      launch_stack<256, 4, kSplitF32>(a, stream, sms, splits, kb_per, ws);
      dim3 grid((N + 1023) / 1024, M);
      if (epi == kSwiGLU) splitk_finalize_kernel<kSwiGLU><<<grid, 256, 0, stream>>>(ws, D, M, N, ldd, splits);
      else if (epi == kStoreF32) splitk_finalize_kernel<kStoreF32><<<grid, 256, 0, stream>>>(ws, D, M, N, ldd, splits);
      else splitk_finalize_kernel<kStoreBf16><<<grid, 256, 0, stream>>>(ws, D, M, N, ldd, splits);
    } else {
      const int bn = choose_bn(M, N, epi);
      if (bn == 0) return LF_NOALLOC_BAD_ARGUMENT;
      if (epi == kSwiGLU) launch_bn<kSwiGLU>(a, bn, stream, sms);
      else if (epi == kStoreF32) launch_bn<kStoreF32>(a, bn, stream, sms);
      else launch_bn<kStoreBf16>(a, bn, stream, sms);
    }
  } catch (...) {
    return LF_NOALLOC_BAD_ARGUMENT;  // tensor-map encoding rejected the operands
  }
  return cudaGetLastError() == cudaSuccess ? LF_NOALLOC_OK : LF_NOALLOC_LAUNCH_FAILED;
}
