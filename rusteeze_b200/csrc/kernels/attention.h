#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {

struct DecodeAttnParams {
  __nv_bfloat16* out;             // [seqs, Hq, D] rows of the output (row stride out_stride)
  int64_t out_stride;
  const __nv_bfloat16* q;         // decode query rows (row stride q_stride)
  int64_t q_stride;
  const __nv_bfloat16* k_cache;   // [blocks, Hkv, 16, D] with block_stride elements between blocks
  const __nv_bfloat16* v_cache;
  int64_t block_stride;
  int num_blocks;                 // cache blocks (page ids outside [0, num_blocks) are rejected)
  const int32_t* seq_lens;        // [seqs]
  const int32_t* block_tables;    // [seqs, bt_stride]
  int64_t bt_stride;
  float* workspace;               // [seqs, Hq, splits, D+2] when num_splits > 1
  int num_seqs, num_q_heads, num_kv_heads, head_dim, num_splits;
  float scale;
  int window;                     // sliding window (0 = none)
  float softcap;                  // 0 = none
  const float* alibi;             // [Hq] ALiBi slopes (nullptr = none): logit += slope * (k_pos - q_pos)
  int* status;
};

struct PrefillAttnParams {
  __nv_bfloat16* out;             // [T, Hq, D] (row stride out_stride)
  int64_t out_stride;
  const __nv_bfloat16* q;         // [T, Hq, D] (row stride q_stride)
  int64_t q_stride;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  int64_t block_stride;
  int num_blocks;
  const int32_t* query_start_loc; // [S+1] over ALL sequences of the batch
  const int32_t* seq_lens;        // [S]
  const int32_t* block_tables;
  int64_t bt_stride;
  int seq_offset;                 // first prefill sequence index
  int num_seqs;                   // prefill sequences
  int max_q_len;
  int num_q_heads, num_kv_heads, head_dim;
  float scale;
  int window;
  float softcap;
  const float* alibi;             // [Hq] ALiBi slopes (nullptr = none)
  int* status;
};

int decode_attention_launch(const DecodeAttnParams& p, cudaStream_t st);
int prefill_attention_launch(const PrefillAttnParams& p, cudaStream_t st);
// tcgen05 FlashAttention prefill (head_dim 128, query heads per kv head dividing 128; not
// ALiBi together with a soft-cap)
bool prefill_tc_supported(const PrefillAttnParams& p);
int prefill_tc_launch(const PrefillAttnParams& p, cudaStream_t st);

}  // namespace rz
