#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {
int argmax_sample_launch(const float* logits, int B, int V, int64_t ld, int64_t* tok, float* lp, int want_lp,
                         cudaStream_t st);
int topk_topp_sample_launch(const float* logits, int B, int V, int64_t ld, const float* temp, const int32_t* topk,
                            const float* topp, const float* minp, const int64_t* seeds, const int64_t* offsets,
                            int64_t* tok, float* lp, cudaStream_t st);
int spec_verify_launch(const float* target, const float* draftl, const int64_t* draft, int B, int k, int V, int64_t ld,
                       const float* temp, const int64_t* seeds, const int64_t* offsets, int64_t* out_tokens,
                       int32_t* n_acc, cudaStream_t st);
}  // namespace rz
