#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {
int spec_verify_launch(const float* target, const float* draftl, const int64_t* draft, int B, int k, int V, int64_t ld,
                       const float* temp, const int64_t* seeds, const int64_t* offsets, int64_t* out_tokens,
                       int32_t* n_acc, cudaStream_t st);
}  // namespace rz

namespace rz {
// ---------------------------------------------------------------- cluster sampler (sampling_cluster.cu)
constexpr int kSampMaxBias = 320;   // logit_bias entries per sequence held on the device
constexpr int kSampMaxStop = 64;    // stop ids masked while fewer than min_tokens were generated

// Device-resident per-sequence sampling state ("slots").
struct SampleSlotTables {
  float* f32;        // [S][8]: temperature, top_p, min_p, repetition, frequency, presence
  int32_t* i32;      // [S][8]: top_k, min_tokens, penalty row (-1: none), n_bias, n_stop
  int32_t* n_gen;    // [S]: tokens generated so far (Philox offset, min_tokens), advanced by the sampler
  int64_t* seed;     // [S]
  uint32_t* cnt;     // [P][ceil(V/2)]: 16-bit output-token counts of penalised slots, two per word
  uint32_t* seen;    // [P][ceil(V/32)]: prompt-token bitmask of penalised slots
  int32_t* bias_tok; // [S][kSampMaxBias]
  float* bias_val;   // [S][kSampMaxBias]
  int32_t* stop_ids; // [S][kSampMaxStop]
};

struct SampleClusterArgs {
  const void* logits;
  int64_t ld;       // row stride in elements
  int R, V, chunk;  // chunk: set by the launcher
  // per-row parameter mode
  const float* temp;
  const int32_t* topk;
  const float* topp;
  const float* minp;
  const int64_t* seeds;
  const int64_t* offsets;
  // slot mode: row_info[r] = slot | (sample index << 16)
  const int32_t* row_info;
  SampleSlotTables st;
  int64_t* tok;
  float* lp;
};

// Uploaded parameters of newly assigned slots (n entries).
struct SampleSlotInit {
  const int32_t* slot;     // [n]
  const float* f32;        // [n][8]
  const int32_t* i32;      // [n][8]
  const int32_t* n_gen;    // [n]
  const int64_t* seed;     // [n]
  const int32_t* bias_tok; // [n][kSampMaxBias]
  const float* bias_val;   // [n][kSampMaxBias]
  const int32_t* stop_ids; // [n][kSampMaxStop]
  const int32_t* tok_off;  // [2n + 1]: prompt / output token ranges of penalised slots in toks
  const int32_t* toks;
};

int sample_cluster_chunk(int V);
int sample_cluster_launch(const SampleClusterArgs& a, bool bf16, bool slots, cudaStream_t st);
int sample_slot_init_launch(const SampleSlotInit& u, int n, const SampleSlotTables& st, int V, cudaStream_t s);
}  // namespace rz
