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
  // cache element format: kKvBf16, or fp8 (kKvE4m3 / kKvE5m2) with k_cache / v_cache pointing
  // at bytes, an element holding value / scale (scales are ignored for bf16)
  int kv_fmt;
  float k_scale, v_scale;
};

constexpr int kKvBf16 = 0, kKvE4m3 = 1, kKvE5m2 = 2;

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
// fp8 cache -> bf16 scratch for the prefill kernels: the blocks of sequences
// [seq_offset, seq_offset + num_seqs) are written densely (sequence by sequence) into
// k_out / v_out [blocks, Hkv, 16, D], and row seq of bt_out [*, bt_out_stride] maps
// each of its pages to its scratch block.  Row offsets are prefix sums of ceil(len / 16).
int kv_dequant_gather_launch(__nv_bfloat16* k_out, __nv_bfloat16* v_out, int32_t* bt_out, int64_t bt_out_stride,
                             const uint8_t* k_cache, const uint8_t* v_cache, int64_t block_stride, int num_blocks,
                             const int32_t* block_tables, int64_t bt_stride, const int32_t* seq_lens,
                             int seq_offset, int num_seqs, int Hkv, int D, int kv_fmt, float k_scale,
                             float v_scale, int64_t out_blocks, int* status, cudaStream_t st);
int prefill_attention_launch(const PrefillAttnParams& p, cudaStream_t st);
// tcgen05 FlashAttention prefill (head_dim 128, query heads per kv head dividing 128; not
// ALiBi together with a soft-cap)
bool prefill_tc_supported(const PrefillAttnParams& p);
int prefill_tc_launch(const PrefillAttnParams& p, cudaStream_t st);

}  // namespace rz
