// Memory-bound elementwise kernels (one pass over HBM each, 16-byte vectors):
//   rms_norm            y = x * rsqrt(mean(x^2) + eps) * (w + offset)
//   fused_add_rms_norm  r += x ; y = rms_norm(r)          (residual updated in place)
//   rope_and_cache      neox RoPE on q (in place) and k of the fused qkv row,
//                       rotated k and raw v written to the paged cache slot
//   act_mul             silu(gate) * up  |  gelu_tanh(gate) * up
// Reference math: RMSNorm with fp32 accumulation (crates/rusteeze-model/src/
// architectures/common.rs:33-45), rotate-half RoPE (common.rs:142-170),
// SwiGLU (common.rs:354-361); the reference's KV write is a no-op
// (crates/rusteeze-tensor/src/cache.rs:484-505).
#include "attention.h"
#include "common.cuh"
#include "elementwise.h"
#include "mxfp8.cuh"

namespace rz {

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

template <int NV>  // 8-element vectors per thread
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  v = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (w == 0) v = warp_sum(v);
  if (threadIdx.x == 0) red[32] = v;
  __syncthreads();
  return red[32];
}

// One CTA per row; blockDim = H / (8*NV).
template <int NV, bool ADD>
__global__ void rms_norm_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                                __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w,
                                int H, float eps, float offset) {
  __shared__ float red[33];
  const size_t row = blockIdx.x;
  const int c0 = threadIdx.x * 8 * NV;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = c0 + j * 8;
    if (c < H) {
      ld8(x + row * H + c, v[j]);
      if (ADD) {
        float r[8];
        ld8(residual + row * H + c, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] += r[i];
        st8(residual + row * H + c, v[j]);
        // the stored (rounded) residual is what later layers see: normalise that
        ld8(residual + row * H + c, v[j]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[j][i] * v[j][i];
    }
  }
  const float inv = rsqrtf(block_sum<NV>(ss, red) / H + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = c0 + j * 8;
    if (c < H) {
      float g[8], o[8];
      ld8(w + c, g);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[j][i] * inv * (g[i] + offset);
      st8(out + row * H + c, o);
    }
  }
}

// RMSNorm (optionally fused with the residual add) whose output goes straight
// to the MXFP8 GEMM operand format: e4m3 values plus one UE8M0 scale per
// 128-column block of the row (written in the GEMM's scale-chunk layout).
// One CTA per row of [0, M_pad); one 8-element vector per thread, so a
// 128-column block is 16 consecutive lanes.  Rows in [M, M_pad) only get the
// neutral scale byte.
template <bool ADD>
__global__ void rms_norm_mxf8_kernel(uint8_t* __restrict__ xq, uint8_t* __restrict__ sfa,
                                     const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                                     const __nv_bfloat16* __restrict__ w, int M, int H, float eps, float offset) {
  __shared__ float red[33];
  const int row = blockIdx.x;
  const int c = threadIdx.x * 8;
  const int kblocks = H / 128;
  uint8_t* chunk = sfa + (static_cast<size_t>(row / 128) * kblocks + c / 128) * kSfChunkBytes + sf_offset(row & 127, 0);
  if (row >= M) {
    if ((threadIdx.x & 15) == 0) *reinterpret_cast<uint32_t*>(chunk) = 0x7f7f7f7fu;
    return;
  }
  const size_t base = static_cast<size_t>(row) * H + c;
  float v[8];
  ld8(x + base, v);
  if (ADD) {
    float r[8];
    ld8(residual + base, r);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] += r[i];
    st8(residual + base, v);
    ld8(residual + base, v);          // normalise the rounded residual, as the bf16 path does
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  const float inv = rsqrtf(block_sum<1>(ss, red) / H + eps);
  float g[8], o[8];
  ld8(w + c, g);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    o[i] = v[i] * inv * (g[i] + offset);
    amax = fmaxf(amax, fabsf(o[i]));
  }
  const unsigned gmask = 0xffffu << (threadIdx.x & 16);
#pragma unroll
  for (int s = 8; s > 0; s >>= 1) amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, s));
  float qinv;
  const uint32_t e = ue8m0_scale(amax, &qinv);
  *reinterpret_cast<uint2*>(xq + base) = pack_e4m3x8(o, qinv);
  if ((threadIdx.x & 15) == 0) *reinterpret_cast<uint32_t*>(chunk) = e * 0x01010101u;
}

int rms_norm_mxf8_launch(uint8_t* xq, uint8_t* sfa, const __nv_bfloat16* x, __nv_bfloat16* residual,
                         const __nv_bfloat16* w, int rows, int H, float eps, float offset, cudaStream_t st) {
  if (rows == 0) return 0;
  if (H % 128 || H > 8192) return -1;
  const int m_pad = (rows + 127) / 128 * 128;
  if (residual)
    rms_norm_mxf8_kernel<true><<<m_pad, H / 8, 0, st>>>(xq, sfa, x, residual, w, rows, H, eps, offset);
  else
    rms_norm_mxf8_kernel<false><<<m_pad, H / 8, 0, st>>>(xq, sfa, x, nullptr, w, rows, H, eps, offset);
  return static_cast<int>(cudaGetLastError());
}

int rms_norm_launch(__nv_bfloat16* out, const __nv_bfloat16* x, __nv_bfloat16* residual,
                    const __nv_bfloat16* w, int rows, int H, float eps, float offset, cudaStream_t st) {
  if (rows == 0) return 0;
  if (H % 8) return -1;
  const int vecs = H / 8;
  // up to 1024 threads, each thread NV vectors
  int nv = (vecs + 1023) / 1024;
  int nv_t = nv <= 1 ? 1 : (nv <= 2 ? 2 : 4);
  const int threads = (vecs + nv_t - 1) / nv_t;
  const int tb = ((threads + 31) / 32) * 32;
#define RZ_LAUNCH_NORM(NV)                                                                              \
  if (residual)                                                                                         \
    rms_norm_kernel<NV, true><<<rows, tb, 0, st>>>(out, x, residual, w, H, eps, offset);                \
  else                                                                                                  \
    rms_norm_kernel<NV, false><<<rows, tb, 0, st>>>(out, x, nullptr, w, H, eps, offset);
  if (nv_t == 1) {
    RZ_LAUNCH_NORM(1)
  } else if (nv_t == 2) {
    RZ_LAUNCH_NORM(2)
  } else {
    RZ_LAUNCH_NORM(4)
  }
#undef RZ_LAUNCH_NORM
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------- RoPE + KV write
// One CTA per token.  Work items: (Hq + Hkv) heads x (D/2)/8 rotation vectors (8 elements of the
// first half with the matching 8 of the second half, 16-byte loads), plus Hkv x D/8 v vectors.
// KVF: cache element format (kKvBf16, or fp8 e4m3 / e5m2 holding value * inv_scale, converted
// with saturation to the largest finite value).
template <int KVF>
__device__ __forceinline__ void st8_kv(void* cache, int64_t elem, const float* v, float inv_scale) {
  if constexpr (KVF == kKvBf16) {
    st8(reinterpret_cast<__nv_bfloat16*>(cache) + elem, v);
  } else {
    const __nv_fp8_interpretation_t fmt = KVF == kKvE4m3 ? __NV_E4M3 : __NV_E5M2;
    uint32_t w[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * k] * inv_scale, v[4 * k + 1] * inv_scale),
                                                   __NV_SATFINITE, fmt);
      const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * k + 2] * inv_scale, v[4 * k + 3] * inv_scale),
                                                   __NV_SATFINITE, fmt);
      w[k] = (lo & 0xffffu) | (hi << 16);
    }
    *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(cache) + elem) = make_uint2(w[0], w[1]);
  }
}

template <int KVF>
__global__ void __launch_bounds__(128) rope_cache_kernel(__nv_bfloat16* __restrict__ qkv, int qkv_stride,
                                                         const int64_t* __restrict__ pos,
                                                         const float* __restrict__ cos_sin, void* __restrict__ kc,
                                                         void* __restrict__ vc, int64_t block_stride,
                                                         const int64_t* __restrict__ slots, int Hq, int Hkv, int D,
                                                         float k_inv_scale, float v_inv_scale) {
  const int t = blockIdx.x;
  __nv_bfloat16* row = qkv + static_cast<size_t>(t) * qkv_stride;
  const int64_t p = pos[t];
  const float* cs = cos_sin + p * D;
  const int half = D / 2;
  const int hv = half / 8;
  const int64_t slot = slots[t];
  const int64_t blk = slot >= 0 ? slot / 16 : 0;
  const int off = slot >= 0 ? static_cast<int>(slot % 16) : 0;
  const int nrot = (Hq + Hkv) * hv;
  for (int i = threadIdx.x; i < nrot; i += blockDim.x) {
    const int h = i / hv, j = (i % hv) * 8;
    __nv_bfloat16* base = row + h * D;
    float x1[8], x2[8], c[8], sn[8], y1[8], y2[8];
    ld8(base + j, x1);
    ld8(base + j + half, x2);
    *reinterpret_cast<float4*>(c) = *reinterpret_cast<const float4*>(cs + j);
    *reinterpret_cast<float4*>(c + 4) = *reinterpret_cast<const float4*>(cs + j + 4);
    *reinterpret_cast<float4*>(sn) = *reinterpret_cast<const float4*>(cs + half + j);
    *reinterpret_cast<float4*>(sn + 4) = *reinterpret_cast<const float4*>(cs + half + j + 4);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      y1[k] = x1[k] * c[k] - x2[k] * sn[k];
      y2[k] = x2[k] * c[k] + x1[k] * sn[k];
    }
    if (h < Hq) {
      st8(base + j, y1);
      st8(base + j + half, y2);
    } else if (slot >= 0) {
      const int64_t dst = blk * block_stride + (static_cast<int64_t>(h - Hq) * 16 + off) * D;
      st8_kv<KVF>(kc, dst + j, y1, k_inv_scale);
      st8_kv<KVF>(kc, dst + j + half, y2, k_inv_scale);
    }
  }
  if (slot >= 0) {
    const int nv = Hkv * D / 8;
    const __nv_bfloat16* vsrc = row + (Hq + Hkv) * D;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      const int h = (i * 8) / D, d = (i * 8) % D;
      const int64_t dst = blk * block_stride + (static_cast<int64_t>(h) * 16 + off) * D + d;
      if constexpr (KVF == kKvBf16) {
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(vc) + dst) =
            *reinterpret_cast<const uint4*>(vsrc + h * D + d);
      } else {
        float x[8];
        ld8(vsrc + h * D + d, x);
        st8_kv<KVF>(vc, dst, x, v_inv_scale);
      }
    }
  }
}

int rope_cache_launch(__nv_bfloat16* qkv, int qkv_stride, const int64_t* pos, const float* cos_sin, void* kc,
                      void* vc, int64_t block_stride, const int64_t* slots, int T, int Hq, int Hkv, int D,
                      int kv_fmt, float k_scale, float v_scale, cudaStream_t st) {
  if (T == 0) return 0;
  if (D % 16 != 0 || qkv_stride % 8 != 0) return -1;
  if (kv_fmt == kKvBf16)
    rope_cache_kernel<kKvBf16><<<T, 128, 0, st>>>(qkv, qkv_stride, pos, cos_sin, kc, vc, block_stride, slots, Hq,
                                                  Hkv, D, 1.f, 1.f);
  else if (kv_fmt == kKvE4m3)
    rope_cache_kernel<kKvE4m3><<<T, 128, 0, st>>>(qkv, qkv_stride, pos, cos_sin, kc, vc, block_stride, slots, Hq,
                                                  Hkv, D, 1.f / k_scale, 1.f / v_scale);
  else if (kv_fmt == kKvE5m2)
    rope_cache_kernel<kKvE5m2><<<T, 128, 0, st>>>(qkv, qkv_stride, pos, cos_sin, kc, vc, block_stride, slots, Hq,
                                                  Hkv, D, 1.f / k_scale, 1.f / v_scale);
  else
    return -1;
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------- act * mul
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  return 0.5f * x * (1.f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}

template <int KIND>
__global__ void act_mul_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x, int I,
                               long total_vec) {
  const long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x;
  if (i >= total_vec) return;
  const int vpr = I / 8;
  const long r = i / vpr;
  const int c = static_cast<int>(i % vpr) * 8;
  float g[8], u[8], o[8];
  ld8(x + r * 2 * I + c, g);
  ld8(x + r * 2 * I + I + c, u);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float a = KIND == 0 ? g[k] / (1.f + __expf(-g[k])) : gelu_tanh(g[k]);
    o[k] = a * u[k];
  }
  st8(out + r * I + c, o);
}

int act_mul_launch(__nv_bfloat16* out, const __nv_bfloat16* x, int rows, int I, int kind, cudaStream_t st) {
  if (rows == 0) return 0;
  if (I % 8) return -1;
  const long total = static_cast<long>(rows) * (I / 8);
  const int tb = 256;
  const int grid = static_cast<int>((total + tb - 1) / tb);
  if (kind == 0)
    act_mul_kernel<0><<<grid, tb, 0, st>>>(out, x, I, total);
  else
    act_mul_kernel<1><<<grid, tb, 0, st>>>(out, x, I, total);
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------- embedding
// out[m] = table[ids[m] - lo] * scale when lo <= ids[m] < hi, else zeros (the rows another
// rank of a vocab-parallel embedding owns; the caller sums the ranks).  Ids outside the
// whole vocabulary are recorded in the status word and give zeros.  One warp per row,
// 16-byte vectors.
__global__ void embedding_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ table,
                                 const int64_t* __restrict__ ids, int M, int H, int64_t lo, int64_t hi, int64_t vocab,
                                 float scale, int* status) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const int lane = threadIdx.x & 31;
  const int64_t id = ids[row];
  if ((id < 0 || id >= vocab) && lane == 0) set_status(status, kBadArgument);
  const bool own = id >= lo && id < hi && id < vocab && id >= 0;
  const __nv_bfloat16* src = table + (own ? (id - lo) : 0) * static_cast<int64_t>(H);
  __nv_bfloat16* dst = out + static_cast<int64_t>(row) * H;
  for (int c = lane * 8; c < H; c += 32 * 8) {
    float v[8];
    if (own) {
      ld8(src + c, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] *= scale;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    st8(dst + c, v);
  }
}

int embedding_launch(__nv_bfloat16* out, const __nv_bfloat16* table, const int64_t* ids, int M, int H, int64_t lo,
                     int64_t hi, int64_t vocab, float scale, int* status, cudaStream_t st) {
  if (M == 0) return 0;
  if (H % 8) return -1;
  const int warps = 8;
  embedding_kernel<<<(M + warps - 1) / warps, warps * 32, 0, st>>>(out, table, ids, M, H, lo, hi, vocab, scale,
                                                                    status);
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------- LayerNorm
// y = (x - mean) * rsqrt(var + eps) * w + b (b optional), fp32 statistics; with a residual,
// r += x first (in place) and the rounded sum is normalised, as in fused_add_rms_norm.
// One CTA per row; blockDim = H / (8 * NV).
template <int NV, bool ADD>
__global__ void layer_norm_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                                  __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w,
                                  const __nv_bfloat16* __restrict__ b, int H, float eps) {
  __shared__ float red[33];
  const size_t row = blockIdx.x;
  const int c0 = threadIdx.x * 8 * NV;
  float v[NV][8];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = c0 + j * 8;
    if (c < H) {
      ld8(x + row * H + c, v[j]);
      if (ADD) {
        float r[8];
        ld8(residual + row * H + c, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] += r[i];
        st8(residual + row * H + c, v[j]);
        ld8(residual + row * H + c, v[j]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[j][i];
    }
  }
  const float mean = block_sum<NV>(s, red) / H;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = c0 + j * 8;
    if (c < H) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[j][i] - mean;
        ss += d * d;
      }
    }
  }
  __syncthreads();   // red is reused by the second reduction
  const float inv = rsqrtf(block_sum<NV>(ss, red) / H + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = c0 + j * 8;
    if (c < H) {
      float g[8], bb[8], o[8];
      ld8(w + c, g);
      if (b) {
        ld8(b + c, bb);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) bb[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[j][i] - mean) * inv * g[i] + bb[i];
      st8(out + row * H + c, o);
    }
  }
}

int layer_norm_launch(__nv_bfloat16* out, const __nv_bfloat16* x, __nv_bfloat16* residual, const __nv_bfloat16* w,
                      const __nv_bfloat16* b, int rows, int H, float eps, cudaStream_t st) {
  if (rows == 0) return 0;
  if (H % 8 || H > 16384) return -1;
  int nv = 1;
  while (H / (8 * nv) > 1024) nv *= 2;
  const int threads = (H / 8 + nv - 1) / nv;
#define RZ_LN(NV)                                                                                           \
  if (residual)                                                                                             \
    layer_norm_kernel<NV, true><<<rows, threads, 0, st>>>(out, x, residual, w, b, H, eps);                  \
  else                                                                                                      \
    layer_norm_kernel<NV, false><<<rows, threads, 0, st>>>(out, x, residual, w, b, H, eps);
  if (nv == 1) {
    RZ_LN(1)
  } else {
    RZ_LN(2)
  }
#undef RZ_LN
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------- KV block copy
// Copies whole KV blocks (all layers) src -> dst inside one cache tensor (copy-on-write).
__global__ void copy_blocks_kernel(uint4* __restrict__ cache, const int32_t* __restrict__ pairs, int64_t vec_per_block) {
  const int b = blockIdx.y;
  const int64_t s = pairs[2 * b], d = pairs[2 * b + 1];
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < vec_per_block;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    cache[d * vec_per_block + i] = cache[s * vec_per_block + i];
}

int copy_blocks_launch(void* cache, const int32_t* pairs, int npairs, int64_t block_bytes, cudaStream_t st) {
  if (npairs == 0) return 0;
  if (block_bytes % 16) return -1;
  dim3 grid(64, npairs);
  copy_blocks_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<uint4*>(cache), pairs, block_bytes / 16);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz
