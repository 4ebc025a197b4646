// Block-scaled FP8 (e4m3) GEMM: D[M,N] = sum_kb (A_kb B_kb^T) * a_scale[kb][m] * b_scale[n/128][kb]
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {
struct Fp8GemmParams {
  int M, N, K;
  int k_splits;           // >= 1 (launcher may reduce it)
  int k_blocks, kb_per_split, m_tiles, n_tiles;   // filled by the launcher
  float* partial;         // [k_splits][M][N] fp32 workspace when k_splits > 1
  int epi;                // kEpiNone | kEpiSiluMul (gate/up rows interleaved in 64-row blocks)
  __nv_bfloat16* D;
  int ldd;
  const float* a_scale;   // [K/128][a_scale_ld >= M]
  int a_scale_ld;
  const float* b_scale;   // [ceil(N/128)][b_scale_ld >= K/128]
  int b_scale_ld;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int ldr;
  int* status;
};
int quant_fp8_act_launch(void* xq, float* xs, const __nv_bfloat16* x, int M, int K, int64_t ldx, int64_t xs_ld,
                         cudaStream_t st);
int gemm_fp8_launch(const Fp8GemmParams& p, const void* A, int lda, const void* B, int ldb, cudaStream_t st);
int fp8_plan_splits(int M, int N, int K);
}  // namespace rz
