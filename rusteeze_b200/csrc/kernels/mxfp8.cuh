// UE8M0 (power-of-two) block scales of the MXFP8 path, shared by the
// quantising producers (activation quant, RMSNorm, GEMM epilogues) and the
// block-scaled GEMM that consumes them.
#pragma once
#include "common.cuh"

namespace rz {

constexpr int kSfChunkBytes = 512;   // scales of 128 rows x 4 K-chunks of 32

// Scale byte position inside a 512-byte chunk for row r (0..127) and K-chunk kc
// (0..3): rows r, r+32, r+64, r+96 share one 16-byte line, which is the order
// in which tcgen05.cp.32x128b.warpx4 spreads a line over TMEM columns.
__host__ __device__ constexpr int sf_offset(int r, int kc) { return (r & 31) * 16 + (r >> 5) * 4 + kc; }

// Power-of-two scale for a block with absolute maximum amax: the smallest 2^e
// with amax / 2^e <= 448 (the e4m3 maximum).  Returns the biased exponent
// byte (UE8M0) and writes 2^-e to *inv.
__device__ __forceinline__ uint32_t ue8m0_scale(float amax, float* inv) {
  int e = -127;
  if (amax > 0.f) {
    const uint32_t bits = __float_as_uint(amax / 448.0f);
    e = static_cast<int>((bits >> 23) & 0xffu) - 127 + ((bits & 0x7fffffu) != 0u ? 1 : 0);
  }
  e = max(-126, min(126, e));
  *inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
  return static_cast<uint32_t>(e + 127);
}

// 8 floats * inv -> 8 e4m3 bytes (saturating)
__device__ __forceinline__ uint2 pack_e4m3x8(const float* v, float inv) {
  uint32_t w[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const __nv_fp8x2_storage_t lo =
        __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i] * inv, v[4 * i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi =
        __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i + 2] * inv, v[4 * i + 3] * inv), __NV_SATFINITE, __NV_E4M3);
    w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  return make_uint2(w[0], w[1]);
}

}  // namespace rz
