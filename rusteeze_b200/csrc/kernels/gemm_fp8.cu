// Block-scaled FP8 GEMM on tcgen05 (kind::f8f6f4) with per-K-block fp32 scale promotion.
#include "common.cuh"
#include "gemm_fp8.h"

namespace rz {
int quant_fp8_act_launch(void*, float*, const __nv_bfloat16*, int, int, int64_t, int64_t, cudaStream_t) { return -100; }
int gemm_fp8_launch(const Fp8GemmParams&, const void*, int, const void*, int, cudaStream_t) { return -100; }
}  // namespace rz
