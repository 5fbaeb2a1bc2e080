#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace moe {

void route(const void* h, const float* wr, const float* bias, int T, int H, int E, int topk, int32_t* ids,
           float* weights, cudaStream_t s);
void align(const int32_t* ids, int T, int topk, int e0, int El, int max_rows, int32_t* groups, int32_t* perm,
           int32_t* slot, cudaStream_t s, int align_rows = 128);
void gather(const void* h, const int32_t* perm, const int32_t* groups, int El, int topk, int H, int max_rows, void* out,
            cudaStream_t s);
void combine(const void* y, const int32_t* slot, const float* w, int T, int topk, int H, void* out, cudaStream_t s);

}  // namespace moe
}  // namespace lf
