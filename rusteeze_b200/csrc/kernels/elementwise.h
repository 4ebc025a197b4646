#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rz {
int rms_norm_launch(__nv_bfloat16* out, const __nv_bfloat16* x, __nv_bfloat16* residual, const __nv_bfloat16* w,
                    int rows, int H, float eps, float offset, cudaStream_t st);
// RMSNorm (+ residual add) emitting the MXFP8 GEMM operand: xq e4m3 [rows, H] and UE8M0
// scale chunks for ceil(rows/128) row blocks.  H % 128 == 0, H <= 8192.
int rms_norm_mxf8_launch(uint8_t* xq, uint8_t* sfa, const __nv_bfloat16* x, __nv_bfloat16* residual,
                         const __nv_bfloat16* w, int rows, int H, float eps, float offset, cudaStream_t st);
// kv_fmt: kKvBf16 (0), kKvE4m3 (1) or kKvE5m2 (2); fp8 caches hold value / scale
int rope_cache_launch(__nv_bfloat16* qkv, int qkv_stride, const int64_t* pos, const float* cos_sin, void* kc,
                      void* vc, int64_t block_stride, const int64_t* slots, int T, int Hq, int Hkv, int D,
                      int kv_fmt, float k_scale, float v_scale, cudaStream_t st);
int act_mul_launch(__nv_bfloat16* out, const __nv_bfloat16* x, int rows, int I, int kind, cudaStream_t st);
int embedding_launch(__nv_bfloat16* out, const __nv_bfloat16* table, const int64_t* ids, int M, int H, int64_t lo,
                     int64_t hi, int64_t vocab, float scale, int* status, cudaStream_t st);
int layer_norm_launch(__nv_bfloat16* out, const __nv_bfloat16* x, __nv_bfloat16* residual, const __nv_bfloat16* w,
                      const __nv_bfloat16* b, int rows, int H, float eps, cudaStream_t st);
int copy_blocks_launch(void* cache, const int32_t* pairs, int npairs, int64_t block_bytes, cudaStream_t st);
}  // namespace rz
