// Speculative-decoding verification (one CTA of 1024 threads per sequence):
// greedy exact match, or standard rejection sampling that preserves the
// target distribution (below).  Row sampling itself is in sampling_cluster.cu.
// Random numbers come from a counter-based Philox4x32-10 stream keyed by
// (seed, step offset, position), implemented from its published description
// (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3",
// SC'11).
#include "common.cuh"
#include "sampling.h"

namespace rz {

constexpr int kSampThreads = 1024;

// ---------------------------------------------------------------- Philox4x32-10 (SC'11)
struct U4 {
  uint32_t x, y, z, w;
};
__device__ __forceinline__ U4 philox_round(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
  const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
  return U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
}
__device__ __forceinline__ U4 philox4x32_10(U4 ctr, uint32_t k0, uint32_t k1) {
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    ctr = philox_round(ctr, k0, k1);
    k0 += W0;
    k1 += W1;
  }
  return ctr;
}
// uniform in (0, 1)
__device__ __forceinline__ float u01(uint32_t v) { return (static_cast<float>(v >> 8) + 0.5f) * (1.0f / 16777216.0f); }

// ---------------------------------------------------------------- block reductions
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < (blockDim.x >> 5) ? red[l] : -INFINITY;
  return warp_max(v);
}
__device__ __forceinline__ float block_sum_f(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < (blockDim.x >> 5) ? red[l] : 0.f;
  return warp_sum(v);
}

// argmax with smallest-index tie break; returns (value, index) to all threads
__device__ __forceinline__ void block_argmax(float& v, int& idx, float* redv, int* redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    redv[w] = v;
    redi[w] = idx;
  }
  __syncthreads();
  v = l < (blockDim.x >> 5) ? redv[l] : -INFINITY;
  idx = l < (blockDim.x >> 5) ? redi[l] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
}

// ---------------------------------------------------------------- speculative verify
// One CTA per sequence.  Rows: target_logits[b*(k+1) + j] for j = 0..k (the
// target's distribution after accepting j draft tokens), draft_logits[b*k + j]
// (the draft's distribution that proposed draft[b, j]).
// Greedy (temp <= 0): accept the longest prefix where draft == target argmax;
// emit the target argmax at the first mismatch, or the bonus token after k.
// Sampled: accept d with probability min(1, p(d)/q(d)); on rejection draw
// from normalise(max(0, p - q)) by Gumbel-max; after k accepts draw the
// bonus token from p.  This is the standard distribution-preserving rule
// (the reference's heuristic `logit[tok] > top * threshold` test at
// crates/rusteeze-engine/src/speculative.rs:316-331 is not).
__device__ __forceinline__ void row_stats(const float* x, int V, float invT, float& m, float& z, float* red) {
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, x[i]);
  m = block_max(mx, red);
  float s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) s += __expf((x[i] - m) * invT);
  z = block_sum_f(s, red);
}

__global__ void __launch_bounds__(kSampThreads)
    spec_verify_kernel(const float* __restrict__ target, const float* __restrict__ draftl, const int64_t* __restrict__ draft,
                       int k, int V, int64_t ld, const float* __restrict__ temp, const int64_t* __restrict__ seeds,
                       const int64_t* __restrict__ offsets, int64_t* __restrict__ out_tokens,
                       int32_t* __restrict__ n_acc) {
  __shared__ float redv[32];
  __shared__ int redi[32];
  const int b = blockIdx.x, tid = threadIdx.x;
  const float T = temp[b];
  const bool greedy = T <= 0.f;
  const float invT = greedy ? 1.f : 1.f / T;
  const uint64_t seed = static_cast<uint64_t>(seeds[b]);
  const uint64_t off = static_cast<uint64_t>(offsets[b]);
  int accepted = 0;
  int64_t* out = out_tokens + static_cast<int64_t>(b) * (k + 1);
  for (int i = tid; i < k + 1; i += blockDim.x) out[i] = -1;
  __syncthreads();
  for (int j = 0; j <= k; ++j) {
    const float* t = target + (static_cast<int64_t>(b) * (k + 1) + j) * ld;
    const int64_t d = j < k ? draft[static_cast<int64_t>(b) * k + j] : -1;
    if (greedy) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int i = tid; i < V; i += blockDim.x)
        if (t[i] > best) { best = t[i]; bi = i; }
      block_argmax(best, bi, redv, redi);
      if (j < k && bi == d) {
        if (tid == 0) out[j] = d;
        ++accepted;
        continue;
      }
      if (tid == 0) out[j] = bi;
      break;
    }
    float mp, zp;
    row_stats(t, V, invT, mp, zp, redv);
    if (j < k) {
      const float* q = draftl + (static_cast<int64_t>(b) * k + j) * ld;
      float mq, zq;
      row_stats(q, V, invT, mq, zq, redv);
      const float pd = __expf((t[d] - mp) * invT) / zp;
      const float qd = __expf((q[d] - mq) * invT) / zq;
      const U4 r = philox4x32_10(U4{0xFFFFFFFFu, static_cast<uint32_t>(off + j), static_cast<uint32_t>((off + j) >> 32),
                                    0x56455249u}, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
      const float U = u01(r.x);
      if (U * qd < pd) {
        if (tid == 0) out[j] = d;
        ++accepted;
        continue;
      }
      // residual draw from max(0, p - q)
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int i = tid; i < V; i += blockDim.x) {
        const float ri = __expf((t[i] - mp) * invT) / zp - __expf((q[i] - mq) * invT) / zq;
        if (ri > 0.f) {
          const U4 rr = philox4x32_10(U4{static_cast<uint32_t>(i), static_cast<uint32_t>(off + j),
                                         static_cast<uint32_t>((off + j) >> 32), 0x52455344u},
                                      static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
          const float key = __logf(ri) - __logf(-__logf(u01(rr.x)));
          if (key > best || (key == best && i < bi)) { best = key; bi = i; }
        }
      }
      block_argmax(best, bi, redv, redi);
      if (tid == 0) out[j] = bi == 0x7fffffff ? d : bi;
      break;
    }
    // bonus token from p
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x) {
      const U4 rr = philox4x32_10(U4{static_cast<uint32_t>(i), static_cast<uint32_t>(off + j),
                                     static_cast<uint32_t>((off + j) >> 32), 0x424F4E55u},
                                  static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
      const float key = (t[i] - mp) * invT - __logf(-__logf(u01(rr.x)));
      if (key > best || (key == best && i < bi)) { best = key; bi = i; }
    }
    block_argmax(best, bi, redv, redi);
    if (tid == 0) out[j] = bi;
  }
  if (tid == 0) n_acc[b] = accepted;
}

int spec_verify_launch(const float* target, const float* draftl, const int64_t* draft, int B, int k, int V, int64_t ld,
                       const float* temp, const int64_t* seeds, const int64_t* offsets, int64_t* out_tokens,
                       int32_t* n_acc, cudaStream_t st) {
  if (B == 0) return 0;
  spec_verify_kernel<<<B, kSampThreads, 0, st>>>(target, draftl, draft, k, V, ld, temp, seeds, offsets, out_tokens,
                                                 n_acc);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz
