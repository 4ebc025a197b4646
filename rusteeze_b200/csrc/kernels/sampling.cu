// Batched token sampling, one CTA (1024 threads) per row of fp32 logits.
//
// Semantics are those of the reference sampler (crates/rusteeze-engine/src/
// sampler.rs:106-179): probabilities p = softmax(x / T); keep the top-k;
// of those keep tokens while the cumulative (un-renormalised) probability of
// the tokens before them is < top_p; renormalise; draw.  min-p additionally
// keeps only p >= min_p * p_max.  Greedy rows take the argmax.
//
// No sort.  With u = (x_max - x) / T >= 0 (p ∝ exp(-u)):
//   pass 1  x_max and Z = sum exp(-u)                              (block reduce)
//   pass 2  2048-bucket histogram of u over [0, 64): count and mass per
//           bucket (warp-aggregated with __match_any_sync, so near-uniform
//           logits do not serialise on a few shared-memory atomics)
//   scan    find the bucket where the running count reaches k or the
//           running mass reaches top_p * Z, whichever comes first
//   pass 3  refine that bucket with another 2048-bucket histogram
//           (resolution 64/2048^2 in u), giving the threshold u*
//   pass 4  Gumbel-max over the kept tokens: argmax(-u_i + g_i), with
//           g_i = -log(-log(U_i)) and U_i from a counter-based Philox4x32-10
//           stream keyed by (seed, step offset, token id).  This draws
//           exactly from the renormalised kept distribution.
// Philox4x32-10 is implemented from its published description (Salmon,
// Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11).
#include "common.cuh"
#include "sampling.h"

namespace rz {

constexpr int kSampThreads = 1024;
constexpr int kBuckets = 2048;
constexpr float kUMax = 64.f;

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

// ---------------------------------------------------------------- greedy
__global__ void __launch_bounds__(kSampThreads) argmax_kernel(const float* __restrict__ logits, int V, int64_t ld,
                                                               int64_t* __restrict__ tok, float* __restrict__ lp,
                                                               int want_lp) {
  __shared__ float redv[32];
  __shared__ int redi[32];
  const float* x = logits + blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = x[i];
    if (v > best) {
      best = v;
      bi = i;
    }
  }
  block_argmax(best, bi, redv, redi);
  float z = 0.f;
  if (want_lp) {
    for (int i = threadIdx.x; i < V; i += blockDim.x) z += __expf(x[i] - best);
    z = block_sum_f(z, redv);
  }
  if (threadIdx.x == 0) {
    tok[blockIdx.x] = bi;
    lp[blockIdx.x] = want_lp ? -__logf(z) : 0.f;
  }
}

// ---------------------------------------------------------------- top-k / top-p / min-p
__device__ __forceinline__ int bucket_of(float u, float lo, float inv_w) {
  int b = static_cast<int>((u - lo) * inv_w);
  return b < 0 ? 0 : (b >= kBuckets ? kBuckets - 1 : b);
}

// Scan 2048 buckets (count, mass) from the top; find the first bucket where
// running count >= k_target or running mass >= m_target.  Warp 0 only.
// Returns bucket index (kBuckets if never reached) and the totals before it.
__device__ void scan_buckets(const int* cnt, const float* mass, long k_target, float m_target, int& out_b,
                             long& cnt_before, float& mass_before) {
  const int lane = threadIdx.x & 31;
  constexpr int per = kBuckets / 32;
  long c = 0;
  float m = 0.f;
  for (int i = 0; i < per; ++i) {
    c += cnt[lane * per + i];
    m += mass[lane * per + i];
  }
  // inclusive scan across lanes
  long ci = c;
  float mi = m;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long oc = __shfl_up_sync(0xffffffffu, ci, o);
    const float om = __shfl_up_sync(0xffffffffu, mi, o);
    if (lane >= o) {
      ci += oc;
      mi += om;
    }
  }
  const bool hit = ci >= k_target || mi >= m_target;
  const unsigned ballot = __ballot_sync(0xffffffffu, hit);
  int b = kBuckets;
  long cb = 0;
  float mb = 0.f;
  if (ballot) {
    const int first = __ffs(ballot) - 1;
    if (lane == first) {
      long cc = ci - c;
      float mm = mi - m;
      for (int i = 0; i < per; ++i) {
        const int bi = lane * per + i;
        // the lane-level sum said the target is reached inside this lane's range; the
        // per-bucket running sum may round differently, so the last bucket is the fallback
        if (cc + cnt[bi] >= k_target || mm + mass[bi] >= m_target || i == per - 1) {
          b = bi;
          break;
        }
        cc += cnt[bi];
        mm += mass[bi];
      }
      cb = cc;
      mb = mm;
    }
    b = __shfl_sync(0xffffffffu, b, first);
    cb = __shfl_sync(0xffffffffu, cb, first);
    mb = __shfl_sync(0xffffffffu, mb, first);
  }
  out_b = b;
  cnt_before = cb;
  mass_before = mb;
}

__device__ __forceinline__ void hist_add(int* cnt, float* mass, int b, float e) {
  // warp-aggregated: lanes hitting the same bucket combine first
  const unsigned grp = __match_any_sync(__activemask(), b);
  if ((grp & (grp - 1)) == 0) {  // alone in its bucket (the common case)
    atomicAdd(&cnt[b], 1);
    atomicAdd(&mass[b], e);
    return;
  }
  const int leader = __ffs(grp) - 1;
  float s = e;
  // sum e over the group via shuffles restricted to members
  unsigned rest = grp;
  float tot = 0.f;
  while (rest) {
    const int src = __ffs(rest) - 1;
    tot += __shfl_sync(grp, s, src);
    rest &= rest - 1;
  }
  if ((threadIdx.x & 31) == leader) {
    atomicAdd(&cnt[b], __popc(grp));
    atomicAdd(&mass[b], tot);
  }
}

__global__ void __launch_bounds__(kSampThreads)
    topk_topp_kernel(const float* __restrict__ logits, int V, int64_t ld, const float* __restrict__ temp,
                     const int32_t* __restrict__ topk, const float* __restrict__ topp,
                     const float* __restrict__ minp, const int64_t* __restrict__ seeds,
                     const int64_t* __restrict__ offsets, int64_t* __restrict__ tok, float* __restrict__ lp) {
  __shared__ int cnt[kBuckets];
  __shared__ float mass[kBuckets];
  __shared__ float redv[32];
  __shared__ int redi[32];
  __shared__ float s_thr[4];
  const int row = blockIdx.x;
  const float* x = logits + row * ld;
  const float T = temp[row];
  const int tid = threadIdx.x;
  // every pass walks the row as 16-byte vectors (4 logits per load, more bytes in flight per
  // thread) when the row allows it, plus a scalar tail
  const bool vec = (ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  const int nv4 = vec ? V / 4 : 0;
  auto for_each = [&](auto&& f) {
#pragma unroll 2
    for (int i4 = tid; i4 < nv4; i4 += blockDim.x) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i4);
      f(4 * i4, v.x);
      f(4 * i4 + 1, v.y);
      f(4 * i4 + 2, v.z);
      f(4 * i4 + 3, v.w);
    }
    for (int i = 4 * nv4 + tid; i < V; i += blockDim.x) f(i, __ldg(x + i));
  };

  // pass 1: max and min (the histogram spans the actual range of u) and, for sampled rows,
  // the normaliser Z = sum exp((x - max) / T) kept as a running (max, sum) pair per thread
  float mx = -INFINITY, mn = INFINITY, zs = 0.f;
  const float invT = T > 0.f ? 1.f / T : 0.f;
  for_each([&](int, float v) {
    if (v > mx) {
      zs = (mx == -INFINITY ? 0.f : zs * __expf((mx - v) * invT)) + 1.f;
      mx = v;
    } else if (mx != -INFINITY) {
      zs += __expf((v - mx) * invT);
    }
    mn = fminf(mn, v);
  });
  const float tmx = mx;
  mx = block_max(mx, redv);
  mn = -block_max(-mn, redv);
  if (T <= 0.f) {  // greedy row inside a sampled batch
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x)
      if (x[i] > best) {
        best = x[i];
        bi = i;
      }
    block_argmax(best, bi, redv, redi);
    float z = 0.f;
    for (int i = tid; i < V; i += blockDim.x) z += __expf(x[i] - mx);
    z = block_sum_f(z, redv);
    if (tid == 0) {
      tok[row] = bi;
      lp[row] = -__logf(z);
    }
    return;
  }
  float z = tmx == -INFINITY ? 0.f : zs * __expf((tmx - mx) * invT);
  z = block_sum_f(z, redv);

  const int k = topk[row] > 0 ? min(topk[row], V) : V;
  const float pth = topp[row];
  const float mp = minp[row];
  // min-p: keep p >= mp * p_max  <=>  u <= -ln(mp)
  const float u_minp = mp > 0.f ? -__logf(mp) : INFINITY;
  // kept set = tokens whose (coarse bucket, fine bucket) index pair is <= (kb1, kb2); the
  // comparison uses the same integer bucket functions as the histograms, so the boundary
  // token is classified exactly as it was counted (a float threshold can round past it)
  int kb1 = kBuckets, kb2 = kBuckets - 1;
  const bool need = (k < V) || (pth < 1.f);
  const float u_range = (mx - mn) * invT;
  const bool clamped = u_range > kUMax;
  const float hi = clamped ? kUMax : (u_range > 0.f ? u_range * 1.0001f : 1.f);
  const float w1 = hi / kBuckets;
  if (need) {
    const float m_target = pth < 1.f ? pth * z : INFINITY;
    // pass 2: coarse histogram over [0, hi)
    for (int i = tid; i < kBuckets; i += blockDim.x) {
      cnt[i] = 0;
      mass[i] = 0.f;
    }
    __syncthreads();
    const float inv_w = 1.f / w1;
    for_each([&](int, float v) {
      const float u = (mx - v) * invT;
      hist_add(cnt, mass, bucket_of(u, 0.f, inv_w), __expf(-u));
    });
    __syncthreads();
    if (tid < 32) {
      int b;
      long cb;
      float mb;
      scan_buckets(cnt, mass, k, m_target, b, cb, mb);
      if (tid == 0) {
        s_thr[0] = static_cast<float>(b);
        s_thr[1] = static_cast<float>(cb);
        s_thr[2] = mb;
      }
    }
    __syncthreads();
    const int b = static_cast<int>(s_thr[0]);
    if (b < kBuckets && !(clamped && b == kBuckets - 1)) {
      const long cb = static_cast<long>(s_thr[1]);
      const float mb = s_thr[2];
      // pass 3: refine bucket b
      const float lo = b * w1;
      const float w2 = w1 / kBuckets;
      __syncthreads();
      for (int i = tid; i < kBuckets; i += blockDim.x) {
        cnt[i] = 0;
        mass[i] = 0.f;
      }
      __syncthreads();
      const float inv_w2 = 1.f / w2;
      for_each([&](int, float v) {
        const float u = (mx - v) * invT;
        if (bucket_of(u, 0.f, inv_w) == b) hist_add(cnt, mass, bucket_of(u, lo, inv_w2), __expf(-u));
      });
      __syncthreads();
      if (tid < 32) {
        int b2;
        long c2;
        float m2;
        scan_buckets(cnt, mass, k - cb, m_target - mb, b2, c2, m2);
        if (tid == 0) s_thr[3] = static_cast<float>(b2 >= kBuckets ? kBuckets - 1 : b2);
      }
      __syncthreads();
      kb1 = b;
      kb2 = static_cast<int>(s_thr[3]);
    }
  }
  const float inv_w1 = 1.f / w1;
  const float lo1 = kb1 < kBuckets ? kb1 * w1 : 0.f;
  const float inv_w2k = 1.f / (w1 / kBuckets);   // bit-identical to pass 3's 1 / w2

  // pass 4: Gumbel-max over kept tokens (and their mass for the logprob)
  const uint64_t seed = static_cast<uint64_t>(seeds[row]);
  const uint64_t off = static_cast<uint64_t>(offsets[row]);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  float kept = 0.f;
  for_each([&](int i, float v) {
    const float u = (mx - v) * invT;
    bool keep = true;
    if (kb1 < kBuckets) {
      const int c1 = bucket_of(u, 0.f, inv_w1);
      keep = c1 < kb1 || (c1 == kb1 && bucket_of(u, lo1, inv_w2k) <= kb2);
    }
    keep = (keep && u <= u_minp) || (u == 0.f);
    if (keep) {
      const float e = __expf(-u);
      kept += e;
      const U4 r = philox4x32_10(U4{static_cast<uint32_t>(i), static_cast<uint32_t>(off),
                                    static_cast<uint32_t>(off >> 32), 0x5A4D504Cu},
                                 static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
      const float g = -__logf(-__logf(u01(r.x)));
      const float key = -u + g;
      if (key > best || (key == best && i < bi)) {
        best = key;
        bi = i;
      }
    }
  });
  block_argmax(best, bi, redv, redi);
  kept = block_sum_f(kept, redv);
  if (tid == 0) {
    tok[row] = bi;
    const float u = (mx - x[bi]) * invT;
    lp[row] = -u - __logf(kept);
  }
}

int argmax_sample_launch(const float* logits, int B, int V, int64_t ld, int64_t* tok, float* lp, int want_lp,
                         cudaStream_t st) {
  if (B == 0) return 0;
  argmax_kernel<<<B, kSampThreads, 0, st>>>(logits, V, ld, tok, lp, want_lp);
  return static_cast<int>(cudaGetLastError());
}

int topk_topp_sample_launch(const float* logits, int B, int V, int64_t ld, const float* temp, const int32_t* topk,
                            const float* topp, const float* minp, const int64_t* seeds, const int64_t* offsets,
                            int64_t* tok, float* lp, cudaStream_t st) {
  if (B == 0) return 0;
  topk_topp_kernel<<<B, kSampThreads, 0, st>>>(logits, V, ld, temp, topk, topp, minp, seeds, offsets, tok, lp);
  return static_cast<int>(cudaGetLastError());
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
