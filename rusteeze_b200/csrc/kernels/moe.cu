// Mixture-of-experts data path (Mixtral-style top-k softmax routing):
//
//   moe_route     router GEMV fused with softmax + top-k: one warp per token
//                 computes the E router logits in fp32 (bf16 inputs), picks
//                 the top-k experts, writes their (renormalised) weights and
//                 counts the tokens of every local expert;
//   moe_permute   turns the counts into expert segments aligned to 128 rows
//                 (so each GEMM M-tile belongs to exactly one expert) and
//                 gathers every (token, slot) pair routed to a local expert
//                 into its expert's segment;
//   grouped GEMMs gate/up with the SiLU(gate)*up epilogue, then down
//                 (gemm_tcgen05 in grouped mode, gemm_bf16.cu);
//   moe_combine   out[t] = sum_k w[t,k] * y[pos(t,k)] (+ residual), fp32.
//
// Nothing here synchronises with the host: segment sizes stay on the device
// and the grouped GEMM reads them, so the whole layer is CUDA-graph capturable.
// With expert parallelism every rank holds all tokens, handles the pairs of
// its experts [e_lo, e_lo + ne) and the partial outputs are summed over ranks.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "gemm_bf16.h"
#include "moe.h"

namespace rz {

constexpr int kMoeMaxExperts = 64;

template <int EMAX>
__global__ void __launch_bounds__(256) moe_route_kernel(MoeRouteParams p) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < p.M; t += gridDim.x * warps) {
    float acc[EMAX];
#pragma unroll
    for (int e = 0; e < EMAX; ++e) acc[e] = 0.f;
    const __nv_bfloat16* x = p.h + static_cast<size_t>(t) * p.ldh;
    for (int c = lane * 8; c < p.H; c += 256) {
      const uint4 xv = *reinterpret_cast<const uint4*>(x + c);
      const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv);
      float xf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(xh[i]);
        xf[2 * i] = f.x;
        xf[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int e = 0; e < EMAX; ++e) {
        if (e < p.E) {
          const uint4 wv = __ldg(reinterpret_cast<const uint4*>(p.wr + static_cast<size_t>(e) * p.H + c));
          const __nv_bfloat162* wh = reinterpret_cast<const __nv_bfloat162*>(&wv);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(wh[i]);
            acc[e] = fmaf(xf[2 * i], f.x, fmaf(xf[2 * i + 1], f.y, acc[e]));
          }
        }
      }
    }
#pragma unroll
    for (int e = 0; e < EMAX; ++e) acc[e] = warp_sum(acc[e]);
    if (lane == 0) {
      float mx = -INFINITY;
      for (int e = 0; e < p.E; ++e) mx = fmaxf(mx, acc[e]);
      float sum = 0.f;
      for (int e = 0; e < p.E; ++e) {
        acc[e] = __expf(acc[e] - mx);
        sum += acc[e];
      }
      uint64_t taken = 0;
      float wsel[8];
      int esel[8];
      float wsum = 0.f;
      for (int j = 0; j < p.topk; ++j) {
        int best = -1;
        float bv = -1.f;
        for (int e = 0; e < p.E; ++e)
          if (!((taken >> e) & 1ull) && acc[e] > bv) { bv = acc[e]; best = e; }
        taken |= 1ull << best;
        wsel[j] = bv / sum;
        esel[j] = best;
        wsum += wsel[j];
      }
      for (int j = 0; j < p.topk; ++j) {
        p.topk_w[t * p.topk + j] = p.renormalize ? wsel[j] / wsum : wsel[j];
        p.topk_id[t * p.topk + j] = esel[j];
        const int le = esel[j] - p.e_lo;
        if (le >= 0 && le < p.ne) atomicAdd(&p.counts[le], 1);
      }
    }
  }
}

// aligned segment starts from the counts (every block recomputes them: ne is small)
__device__ __forceinline__ void segment_starts(const int* counts, int ne, int* s_off) {
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < ne; ++e) {
      s_off[e] = o;
      o += (counts[e] + 127) / 128 * 128;
    }
    s_off[ne] = o;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(256) moe_permute_kernel(MoePermuteParams p) {
  __shared__ int s_off[kMoeMaxExperts + 1];
  segment_starts(p.counts, p.ne, s_off);
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e <= p.ne; e += blockDim.x) p.grp_off[e] = s_off[e];
    for (int e = threadIdx.x; e < p.ne; e += blockDim.x) p.grp_end[e] = s_off[e] + p.counts[e];
  }
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pairs = p.M * p.topk;
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < pairs; i += gridDim.x * warps) {
    const int le = p.topk_id[i] - p.e_lo;
    int pos = -1;
    if (le >= 0 && le < p.ne) {
      if (lane == 0) pos = s_off[le] + atomicAdd(&p.fill[le], 1);
      pos = __shfl_sync(0xffffffffu, pos, 0);
      const uint4* src = reinterpret_cast<const uint4*>(p.h + static_cast<size_t>(i / p.topk) * p.ldh);
      uint4* dst = reinterpret_cast<uint4*>(p.x_perm + static_cast<size_t>(pos) * p.H);
      for (int c = lane; c < p.H / 8; c += 32) dst[c] = src[c];
    }
    if (lane == 0) p.pos_of[i] = pos;
  }
}

// one thread per 8 output columns of one token
__global__ void moe_combine_kernel(MoeCombineParams p) {
  const int vec = p.H / 8;
  const long idx = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long>(p.M) * vec) return;
  const int t = static_cast<int>(idx / vec);
  const int c = static_cast<int>(idx % vec) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < p.topk; ++j) {
    const int pos = p.pos_of[t * p.topk + j];
    if (pos < 0) continue;
    const float w = p.topk_w[t * p.topk + j];
    const uint4 u = *reinterpret_cast<const uint4*>(p.y + static_cast<size_t>(pos) * p.ldy + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      acc[2 * i] = fmaf(w, f.x, acc[2 * i]);
      acc[2 * i + 1] = fmaf(w, f.y, acc[2 * i + 1]);
    }
  }
  if (p.residual) {
    const uint4 u = *reinterpret_cast<const uint4*>(p.residual + static_cast<size_t>(t) * p.H + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
  uint4 o;
  __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
  *reinterpret_cast<uint4*>(p.out + static_cast<size_t>(t) * p.H + c) = o;
}

int moe_route_launch(const MoeRouteParams& p, cudaStream_t st) {
  if (p.E > 32 || p.topk > 8 || p.H % 256 != 0) return -1;
  const int blocks = (p.M + 7) / 8 < 1024 ? (p.M + 7) / 8 : 1024;
  if (p.M == 0) return 0;
  if (p.E <= 8)
    moe_route_kernel<8><<<blocks, 256, 0, st>>>(p);
  else if (p.E <= 16)
    moe_route_kernel<16><<<blocks, 256, 0, st>>>(p);
  else
    moe_route_kernel<32><<<blocks, 256, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int moe_permute_launch(const MoePermuteParams& p, cudaStream_t st) {
  if (p.ne > kMoeMaxExperts || p.H % 8 != 0) return -1;
  const int pairs = p.M * p.topk;
  int blocks = (pairs + 7) / 8;
  blocks = blocks < 1 ? 1 : (blocks > 1024 ? 1024 : blocks);
  moe_permute_kernel<<<blocks, 256, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int moe_combine_launch(const MoeCombineParams& p, cudaStream_t st) {
  if (p.H % 8 != 0) return -1;
  const long threads = static_cast<long>(p.M) * (p.H / 8);
  if (threads == 0) return 0;
  moe_combine_kernel<<<static_cast<int>((threads + 255) / 256), 256, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz
