// Word-level primitives of the low-latency all-reduce protocol (see
// allreduce_ll.cu): every 8-byte word carries two bf16 values and the epoch of
// the operation and is written by one store, so a reader that sees the epoch
// sees the data.  Shared by the standalone all-reduce kernel and the GEMM whose
// epilogue runs the protocol itself.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace lf {
namespace ar {

__device__ __forceinline__ void st_word(uint2* p, uint32_t data, uint32_t ep) {
  asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(ep) : "memory");
}

__device__ __forceinline__ void st_word_mc(uint2* p, uint32_t data, uint32_t ep) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(ep) : "memory");
}

__device__ __forceinline__ uint2 ld_word(const uint2* p) {
  uint2 v;
  asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// Polls one inbox word until it carries epoch `ep`; false after recording a
// timeout (or when another wait already failed).
__device__ __forceinline__ bool poll_word(const uint2* p, uint32_t ep, uint32_t* data) {
  uint2 v = ld_word(p);
  if (v.y != ep) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    do {
      if ((++spins & 255u) == 0) {
        if (error_pending()) return false;
        if (globaltimer_ns() - t0 > wait_limit_ns()) {
          set_error(kErrPeerTimeout, 0x11ull);
          return false;
        }
      }
      v = ld_word(p);
    } while (v.y != ep);
  }
  *data = v.x;
  return true;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack2(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}

}  // namespace ar
}  // namespace lf
