#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lf {
namespace attn {

struct DecodeArgs {
  const __nv_bfloat16* q;      // token rows, Q heads first; row stride q_ld
  int64_t q_ld;
  __nv_bfloat16* out;          // [T, Hq * D]; row stride out_ld
  int64_t out_ld;
  const int32_t* tok_index;    // [rows] token row of each decode row
  const int32_t* seq_lens;     // [rows] KV length including the new token
  const int32_t* block_table;  // [rows, bt_stride] physical page ids
  int64_t bt_stride;
  int rows, Hq, Hkv, D, page, num_pages, splits;
  float scale_log2;            // (1 / sqrt(D)) * log2(e)
  float* part_o;               // [rows, Hq, splits, D] workspace when splits > 1
  float* part_lse;             // [rows, Hq, splits]
};

struct PrefillArgs {
  const __nv_bfloat16* q;
  int64_t q_ld;
  __nv_bfloat16* out;
  int64_t out_ld;
  const int32_t* q_start;      // [rows + 1] CSR query offsets (token rows)
  const int32_t* seq_lens;     // [rows] KV length including this chunk
  const int32_t* block_table;  // [rows, bt_stride]
  int64_t bt_stride;
  int rows, Hq, Hkv, D, page, num_pages, max_q_len;
  float scale_log2;
  int q_rows;                  // rows of q (token rows of this step's prefill part)
  int* progress;               // optional (null in production): per-CTA progress codes, host-visible memory
};

int decode_splits(int rows, int Hkv, int max_seq, int num_sms);
void decode(const DecodeArgs& a, const void* kcache, const void* vcache, cudaStream_t stream);
// Prefill attention: the tcgen05 kernel (attention_tc.cu) for GQA groups of
// 1, 2, 4, 8 or 16 heads, else (or with LUNAFLUX_PREFILL_MMA_SYNC set) the
// mma.sync kernel.
void prefill(const PrefillArgs& a, const void* kcache, const void* vcache, cudaStream_t stream);
bool prefill_tc_supported(const PrefillArgs& a);
void prefill_tc(const PrefillArgs& a, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream);

}  // namespace attn
}  // namespace lf
