#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace ew {

// Per-row sampling parameters, laid out for a single H2D copy per step.
struct SampleParams {
  int32_t mode;          // 0 greedy, 1 stochastic
  int32_t top_k;         // <= 0: disabled
  float temperature;     // > 0 for stochastic rows
  float top_p;           // (0, 1]; >= 1 disables
  uint64_t seed;         // non-zero request seed
  int64_t sample_index;  // index of the token being drawn (output position)
};
static_assert(sizeof(SampleParams) == 32, "SampleParams is a 32-byte wire record");

// fwd / prev: forwarded decode tokens (see elementwise.cu); null for none.
void embed(int32_t* ids, const void* table, void* out, int T, int H, int vocab, cudaStream_t s,
           const int32_t* fwd = nullptr, int fwd_first = 0, int nfwd = 0, const int32_t* prev = nullptr,
           int nprev = 0);
// rows: gathered form (output row i from input row rows[i] of in_rows; no residual write-back).
void rmsnorm(const void* x, void* residual, const void* w, void* out, int T, int H, float eps, cudaStream_t s,
             const int32_t* rows = nullptr, int in_rows = 0);
void rope_kv_write(void* qkv, int64_t ld, const int32_t* positions, const int32_t* slots, const void* cos_sin,
                   void* kcache, void* vcache, int T, int Hq, int Hkv, int D, int page, int max_pos,
                   int64_t num_slots, cudaStream_t s);
void swiglu(const void* gu, void* out, int T, int F, cudaStream_t s);
void argmax(const float* logits, int64_t ld, int R, int V, int32_t* out, int32_t* status, cudaStream_t s);
void argmax_keys(const float* logits, int64_t ld, int R, int V, int id_offset, unsigned long long* keys,
                 cudaStream_t s);
void keys_to_tokens(const unsigned long long* keys, int R, int ranks, int32_t* out, cudaStream_t s);
// Vocabulary-parallel sampling: each shard's kc largest keys plus a status
// word per row (out [R][kc + 1]); then the draw over all shards' candidates
// (keys [ranks][R][kc + 1]), exact for rows with 0 < top_k <= kc.
void topk_keys(const float* logits, int64_t ld, int R, int V, int id_offset, int kc, unsigned long long* out,
               cudaStream_t s);
void sample_keys(const unsigned long long* keys, int R, int ranks, int kc, const SampleParams* params, int32_t* out,
                 int32_t* status, cudaStream_t s);
void sample(const float* logits, int64_t ld, int R, int V, const SampleParams* params, int32_t* out, int32_t* status,
            cudaStream_t s);
double host_counter_unit(uint64_t seed, int64_t idx);

}  // namespace ew
}  // namespace lf
