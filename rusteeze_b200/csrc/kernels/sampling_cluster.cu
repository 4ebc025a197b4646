// Token sampling with one thread-block cluster per row of logits.
//
// The row (bf16 or fp32, up to ~400K entries) is split over the 8 CTAs of a
// cluster; each CTA reads its slice from HBM exactly once into shared memory,
// and every later pass (penalties, max, normaliser, two histogram levels,
// the draw) runs on shared memory.  The CTAs combine their partial results
// through distributed shared memory (DSMEM) at cluster barriers, so a row
// costs one HBM read instead of one per pass.  Semantics are those of the
// reference sampler (crates/rusteeze-engine/src/sampler.rs:56-244 and the
// penalties of simd_ops.rs:89-119):
//
//   penalties  repetition (tokens seen in the prompt or the output: x/r when
//              x > 0, x*r otherwise), then frequency and presence over the
//              output counts: x -= f*count + p*(count > 0);
//   bias       x += logit_bias[t];
//   min_tokens the stop ids (EOS + stop_token_ids) are -inf while fewer than
//              min_tokens tokens were generated;
//   greedy     T <= 0 or top_k == 1: argmax, logprob from the raw softmax;
//   otherwise  e = exp((x - max) / T) = p / p_max; keep the top-k, then the
//              tokens whose preceding (un-renormalised) mass is < top_p, and
//              e >= min_p; draw one token from the kept mass by inverse CDF with
//              one uniform number from a counter-based Philox4x32-10 stream keyed
//              by (seed, tokens generated so far).
//
// The top-k / top-p threshold is found without a sort by radix selection on
// the IEEE bits of e (a positive float's bit pattern orders like its value):
// a 2048-bucket histogram of count and mass on bits [30:20] (exponent + 3
// mantissa bits), then a second 2048-bucket level on bits [19:9] inside the
// bucket where the running count or mass crosses the target.  Tokens whose
// first 22 key bits tie with the boundary are kept or dropped together.  Every
// token of a bucket shares its exponent, so a bucket's mass is accumulated as
// an integer sum of 21-bit mantissas: lanes of a warp that hit the same bucket
// are combined with one match and one integer warp reduction, and their
// leader does one shared-memory add.
//
// The draw walks the kept mass in (thread, stride) order rather than token
// order: thread t of a CTA owns tokens t, t + 512, ...; per-thread kept sums,
// a CTA total per cluster rank, and one uniform u pick the CTA, then the
// thread, then the token where the running mass crosses u times the total.
// Any fixed order gives the same distribution.
//
// Parameters come either from per-row arrays, or (slot mode) from
// device-resident per-sequence tables indexed by a slot id per row: the host
// uploads a sequence's parameters once, and this kernel advances the slot's
// generated-token counter and its penalty counts itself after each draw, so a
// pipelined engine never has to send per-step sampling state.
//
// Philox4x32-10 is implemented from its published description (Salmon,
// Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11).
#include <cooperative_groups.h>

#include "common.cuh"
#include "sampling.h"

namespace rz {
namespace cg = cooperative_groups;

namespace {

constexpr int kCl = 8;        // CTAs per row (portable cluster size)
constexpr int kThr = 512;     // threads per CTA
constexpr int kHB = 2048;     // histogram buckets per level

struct P4 {
  uint32_t x, y, z, w;
};
__device__ __forceinline__ P4 ph_round(P4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
  const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
  return P4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
}
__device__ __forceinline__ P4 philox10(P4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    c = ph_round(c, k0, k1);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}
__device__ __forceinline__ float unit_open(uint32_t v) {  // uniform in (0, 1)
  return (static_cast<float>(v >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

// (value, index) max with the smaller index winning ties
__device__ __forceinline__ void amax_merge(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}
__device__ __forceinline__ void block_amax(float& v, int& i, float* rv, int* ri) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax_merge(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    rv[w] = v;
    ri[w] = i;
  }
  __syncthreads();
  v = l < kThr / 32 ? rv[l] : -INFINITY;
  i = l < kThr / 32 ? ri[l] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax_merge(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
}
__device__ __forceinline__ float block_sum(float v, float* rv) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) rv[w] = v;
  __syncthreads();
  v = l < kThr / 32 ? rv[l] : 0.f;
  return warp_sum(v);
}

// Histogram add: lanes of a warp with the same bucket are combined (count by popcount,
// mass as an integer sum of mantissas) and their leader adds once.  `mfx` is the token's
// 21-bit mantissa with the implicit 1 (1.m * 2^20); a bucket's tokens share an exponent.
__device__ __forceinline__ void hist_add(int* cnt, unsigned long long* mass, int b, uint32_t mfx) {
  const unsigned grp = __match_any_sync(__activemask(), b);
  const uint32_t tot = __reduce_add_sync(grp, mfx);
  if ((threadIdx.x & 31) == __ffs(grp) - 1) {
    atomicAdd(&cnt[b], __popc(grp));
    atomicAdd(&mass[b], static_cast<unsigned long long>(tot));
  }
}
__device__ __forceinline__ uint32_t mant_fx(uint32_t u) { return ((u & 0x7fffffu) >> 3) | (1u << 20); }

// CTA 0 only: sums the cluster's histograms into its own, then warp 0 walks the buckets
// from the largest key down and finds the first one where the running count reaches
// k_target or the running mass reaches m_target.  `scale(b)` turns bucket b's integer
// mass into e units.  Writes (bucket or -1, count before) and (mass before) to sel.
template <typename Scale>
__device__ void merge_and_scan(cg::cluster_group& cl, int* hcnt, unsigned long long* hm, float* hf, long k_target,
                               float m_target, Scale scale, int* sel_i, float* sel_f) {
  for (int b = threadIdx.x; b < kHB; b += kThr) {
    int c = 0;
    unsigned long long m = 0;
#pragma unroll
    for (int r = 0; r < kCl; ++r) {
      c += *cl.map_shared_rank(hcnt + b, r);
      m += *cl.map_shared_rank(hm + b, r);
    }
    hcnt[b] = c;
    hf[b] = static_cast<float>(m) * scale(b);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    constexpr int per = kHB / 32;
    // lane l owns the descending-order range [l*per, (l+1)*per): bucket kHB-1-i
    long c = 0;
    float m = 0.f;
    for (int i = 0; i < per; ++i) {
      const int b = kHB - 1 - (lane * per + i);
      c += hcnt[b];
      m += hf[b];
    }
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
    const unsigned hit = __ballot_sync(0xffffffffu, ci >= k_target || mi >= m_target);
    if (lane == 0) {
      sel_i[0] = -1;
      sel_i[1] = 0;
      sel_f[0] = 0.f;
    }
    __syncwarp();
    if (hit) {
      const int first = __ffs(hit) - 1;
      if (lane == first) {
        long cc = ci - c;
        float mm = mi - m;
        int bsel = kHB - 1 - (lane * per + per - 1);
        for (int i = 0; i < per; ++i) {
          const int b = kHB - 1 - (lane * per + i);
          // the lane total said the target is reached in this range; rounding of the
          // per-bucket sums may differ, so the range's last bucket is the fallback
          if (cc + hcnt[b] >= k_target || mm + hf[b] >= m_target || i == per - 1) {
            bsel = b;
            break;
          }
          cc += hcnt[b];
          mm += hf[b];
        }
        sel_i[0] = bsel;
        sel_i[1] = static_cast<int>(cc);
        sel_f[0] = mm;
      }
    }
  }
  __syncthreads();
}

template <bool BF16>
__device__ __forceinline__ float load1(const void* row, int64_t i) {
  if (BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(row)[i]);
  return static_cast<const float*>(row)[i];
}

// 2^k for an integer exponent (the mass scale of a histogram bucket)
__device__ __forceinline__ float pow2i(int k) { return ldexpf(1.f, k); }

}  // namespace

template <bool BF16, bool SLOTS>
__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kThr) sample_cluster_kernel(SampleClusterArgs a) {
  cg::cluster_group cl = cg::this_cluster();
  const int cr = static_cast<int>(cl.block_rank());
  const int row = blockIdx.x / kCl;
  const int tid = threadIdx.x;
  extern __shared__ __align__(16) float xs[];
  __shared__ int hcnt[kHB];
  __shared__ unsigned long long hm[kHB];
  __shared__ float hf[kHB];
  __shared__ float tsum[kThr];
  __shared__ float rv[32];
  __shared__ int ri[32];
  // per-CTA partial results that the other CTAs read through DSMEM
  __shared__ float c_max, c_sum, c_kept;
  __shared__ int c_arg;
  // CTA 0's threshold selections (one set per level), read by every CTA
  __shared__ int sel_i[2][2];
  __shared__ float sel_f[2][1];

  // ---------------------------------------------------------------- parameters
  float T, top_p, min_p, rep = 1.f, freq = 0.f, pres = 0.f;
  int top_k, pen = -1, nbias = 0, nstop = 0, slot = 0, jsub = 0;
  uint64_t seed, off;
  bool mask_stops = false;
  if (SLOTS) {
    const int info = a.row_info[row];
    slot = info & 0xffff;
    jsub = info >> 16;
    const float* f = a.st.f32 + slot * 8;
    const int32_t* q = a.st.i32 + slot * 8;
    T = f[0];
    top_p = f[1];
    min_p = f[2];
    rep = f[3];
    freq = f[4];
    pres = f[5];
    top_k = q[0];
    pen = q[2];
    nbias = q[3];
    nstop = q[4];
    const int ngen = a.st.n_gen[slot];
    mask_stops = ngen < q[1];
    seed = static_cast<uint64_t>(a.st.seed[slot]) + 7919ull * static_cast<uint64_t>(jsub);
    off = static_cast<uint64_t>(ngen);
  } else {
    T = a.temp[row];
    top_p = a.topp[row];
    min_p = a.minp[row];
    top_k = a.topk[row];
    seed = static_cast<uint64_t>(a.seeds[row]);
    off = static_cast<uint64_t>(a.offsets[row]);
  }
  const int V = a.V;
  const bool greedy = !(T > 0.f) || top_k == 1;
  const int lo = cr * a.chunk;
  const int n = max(0, min(a.chunk, V - lo));
  const size_t esz = BF16 ? 2 : 4;
  const char* rowp = static_cast<const char*>(a.logits) + static_cast<size_t>(row) * a.ld * esz;
  const int64_t cw = (V + 1) / 2, sw = (V + 31) / 32;

  // ---------------------------------------------------------------- 1. load (+ penalties), running max
  auto penal = [&](int t, float x) -> float {
    const uint32_t w = a.st.cnt[static_cast<int64_t>(pen) * cw + (t >> 1)];
    const uint32_t c = (t & 1) ? (w >> 16) : (w & 0xffffu);
    const bool seen = (a.st.seen[static_cast<int64_t>(pen) * sw + (t >> 5)] >> (t & 31)) & 1u;
    if (rep != 1.f && (c > 0 || seen)) x = x > 0.f ? x / rep : x * rep;
    return x - freq * static_cast<float>(c) - (c > 0 ? pres : 0.f);
  };
  float mv = -INFINITY;
  int mi = 0x7fffffff;
  const bool vec = ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0) && ((a.ld * esz) % 16 == 0);
  constexpr int VE = BF16 ? 8 : 4;   // elements per 16-byte load
  const int nvec = vec ? n / VE : 0;
  for (int v = tid; v < nvec; v += kThr) {
    const uint4 raw = *reinterpret_cast<const uint4*>(rowp + (static_cast<size_t>(lo) + v * VE) * esz);
    float x[VE];
    if (BF16) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f2 = __bfloat1622float2(h[k]);
        x[2 * k] = f2.x;
        x[2 * k + 1] = f2.y;
      }
    } else {
      const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
      for (int k = 0; k < VE; ++k) x[k] = f[k];
    }
    if (SLOTS && pen >= 0) {
#pragma unroll
      for (int k = 0; k < VE; ++k) x[k] = penal(lo + v * VE + k, x[k]);
    }
#pragma unroll
    for (int k = 0; k < VE; ++k) amax_merge(mv, mi, x[k], lo + v * VE + k);
#pragma unroll
    for (int k = 0; k < VE; k += 4)
      *reinterpret_cast<float4*>(xs + v * VE + k) = make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]);
  }
  for (int i = nvec * VE + tid; i < n; i += kThr) {
    float x = load1<BF16>(rowp, lo + i);
    if (SLOTS && pen >= 0) x = penal(lo + i, x);
    amax_merge(mv, mi, x, lo + i);
    xs[i] = x;
  }
  if (SLOTS && (nbias > 0 || (mask_stops && nstop > 0))) {
    // sparse fixups inside this CTA's slice (bias ids are distinct: a map's keys; a stop id
    // listed twice writes -inf twice), then the slice's max again
    __syncthreads();
    for (int k = tid; k < nbias; k += kThr) {
      const int t = a.st.bias_tok[slot * kSampMaxBias + k];
      if (t >= lo && t < lo + n) xs[t - lo] += a.st.bias_val[slot * kSampMaxBias + k];
    }
    __syncthreads();
    if (mask_stops) {
      for (int k = tid; k < nstop; k += kThr) {
        const int t = a.st.stop_ids[slot * kSampMaxStop + k];
        if (t >= lo && t < lo + n) xs[t - lo] = -INFINITY;
      }
    }
    __syncthreads();
    mv = -INFINITY;
    mi = 0x7fffffff;
    for (int i = tid; i < n; i += kThr) amax_merge(mv, mi, xs[i], lo + i);
  }

  // ---------------------------------------------------------------- 2. max / argmax over the cluster
  block_amax(mv, mi, rv, ri);
  if (tid == 0) {
    c_max = mv;
    c_arg = mi;
  }
  cl.sync();
  float M = -INFINITY;
  int arg = 0x7fffffff;
#pragma unroll
  for (int r = 0; r < kCl; ++r) amax_merge(M, arg, *cl.map_shared_rank(&c_max, r), *cl.map_shared_rank(&c_arg, r));
  if (arg == 0x7fffffff) arg = 0;   // every logit -inf (fully masked row)

  // ---------------------------------------------------------------- 3. normaliser; e = exp((x - M) / T) in place
  const float invT = greedy ? 1.f : 1.f / T;
  const float s2 = invT * 1.4426950408889634f;   // exp(y) = exp2(y * log2 e)
  float z = 0.f;
  if (greedy) {
    for (int i = tid; i < n; i += kThr) z += exp2f((xs[i] - M) * s2);
  } else {
    for (int i = tid; i < n; i += kThr) {
      const float e = exp2f((xs[i] - M) * s2);
      xs[i] = e;
      z += e;
    }
  }
  z = block_sum(z, rv);
  if (tid == 0) c_sum = z;
  cl.sync();
  float Z = 0.f;
#pragma unroll
  for (int r = 0; r < kCl; ++r) Z += *cl.map_shared_rank(&c_sum, r);

  auto post_update = [&](int tok) {   // CTA 0, thread 0: the slot's counters after a draw
    if (SLOTS && jsub == 0) {
      a.st.n_gen[slot] += 1;
      if (pen >= 0) {
        uint32_t* w = a.st.cnt + static_cast<int64_t>(pen) * cw + (tok >> 1);
        const uint32_t sh = (tok & 1) * 16;
        if (((*w >> sh) & 0xffffu) != 0xffffu) *w += 1u << sh;
      }
    }
  };
  if (greedy) {
    if (cr == 0 && tid == 0) {
      a.tok[row] = arg;
      a.lp[row] = -__logf(Z);
      post_update(arg);
    }
    cl.sync();   // no CTA leaves while a peer may still read its shared memory
    return;
  }

  // ---------------------------------------------------------------- 4. top-k / top-p threshold (radix select on e)
  const int k = top_k > 0 ? min(top_k, V) : V;
  const bool trunc = k < V || top_p < 1.f;
  int kb1 = -1, kb2 = 0;   // kept: key1 > kb1, or key1 == kb1 and key2 >= kb2 (kb1 < 0: all)
  if (trunc) {
    const float m_target = top_p < 1.f ? top_p * Z : INFINITY;
    for (int b = tid; b < kHB; b += kThr) {
      hcnt[b] = 0;
      hm[b] = 0ull;
    }
    __syncthreads();
    for (int i = tid; i < n; i += kThr) {
      const uint32_t u = __float_as_uint(xs[i]);
      if (u >= 0x00800000u) hist_add(hcnt, hm, static_cast<int>(u >> 20), mant_fx(u));   // normal e > 0
    }
    __syncthreads();
    cl.sync();
    // bucket b holds exponent b >> 3: mass = sum(1.m * 2^20) * 2^(E - 127 - 20)
    if (cr == 0)
      merge_and_scan(cl, hcnt, hm, hf, k, m_target, [](int b) { return pow2i((b >> 3) - 147); }, sel_i[0],
                     sel_f[0]);
    cl.sync();
    const int b1 = *cl.map_shared_rank(&sel_i[0][0], 0);
    const long cb = *cl.map_shared_rank(&sel_i[0][1], 0);
    const float mb = *cl.map_shared_rank(&sel_f[0][0], 0);
    if (b1 >= 0) {
      for (int b = tid; b < kHB; b += kThr) {
        hcnt[b] = 0;
        hm[b] = 0ull;
      }
      __syncthreads();
      for (int i = tid; i < n; i += kThr) {
        const uint32_t u = __float_as_uint(xs[i]);
        if (static_cast<int>(u >> 20) == b1) hist_add(hcnt, hm, static_cast<int>((u >> 9) & 0x7ffu), mant_fx(u));
      }
      __syncthreads();
      cl.sync();
      const float sc = pow2i((b1 >> 3) - 147);
      if (cr == 0)
        merge_and_scan(cl, hcnt, hm, hf, k - cb, m_target - mb, [sc](int) { return sc; }, sel_i[1], sel_f[1]);
      cl.sync();
      const int b2 = *cl.map_shared_rank(&sel_i[1][0], 0);
      kb1 = b1;
      kb2 = b2 < 0 ? 0 : b2;
    }
  }

  // ---------------------------------------------------------------- 5. draw by inverse CDF over the kept mass
  auto kept_e = [&](int i) -> float {
    const float e = xs[i];
    const uint32_t u = __float_as_uint(e);
    bool keep = e > 0.f;
    if (kb1 >= 0) {
      const int key1 = static_cast<int>(u >> 20);
      keep = keep && (key1 > kb1 || (key1 == kb1 && static_cast<int>((u >> 9) & 0x7ffu) >= kb2));
    }
    keep = (keep && e >= min_p) || e == 1.f;   // the most likely token is always kept
    return keep ? e : 0.f;
  };
  float ts = 0.f;
  for (int i = tid; i < n; i += kThr) ts += kept_e(i);
  tsum[tid] = ts;
  const float kept = block_sum(ts, rv);   // starts with a barrier: tsum is complete after it
  if (tid == 0) {
    c_kept = kept;
    c_arg = arg;                           // replaced by the drawn token in the owning CTA
    if (cr == 0) {
      a.tok[row] = arg;                    // (nothing kept at all: the argmax stands)
      a.lp[row] = 0.f;
    }
  }
  cl.sync();
  float ctot[kCl];
  float total = 0.f;
#pragma unroll
  for (int r = 0; r < kCl; ++r) {
    ctot[r] = *cl.map_shared_rank(&c_kept, r);
    total += ctot[r];
  }
  // one uniform per row and step
  const P4 rnd = philox10(P4{0x53414D50u, static_cast<uint32_t>(off), static_cast<uint32_t>(off >> 32), 0x5A4D504Cu},
                          static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  const float target = unit_open(rnd.x) * total;
  // the CTA whose running total crosses the target (the last CTA with mass takes rounding)
  int owner = -1, last = -1;
  float before = 0.f, acc = 0.f;
#pragma unroll
  for (int r = 0; r < kCl; ++r) {
    if (ctot[r] > 0.f) {
      last = r;
      if (owner < 0 && acc + ctot[r] > target) {
        owner = r;
        before = acc;
      }
    }
    acc += ctot[r];
  }
  if (owner < 0 && last >= 0) {
    owner = last;
    before = acc - ctot[last];
  }
  if (owner < 0) owner = 0;                    // nothing kept: the argmax below
  if (cr == owner) {
    // inclusive prefix of the per-thread sums in thread order; thread i's range is
    // [P(i-1), P(i)) with P(i-1) taken from its neighbour, so ranges neither overlap nor gap
    __shared__ float wsum[kThr / 32];
    __shared__ int last_t;
    const int w = tid >> 5, l = tid & 31;
    const float mine_sum = tsum[tid];
    if (tid == 0) last_t = -1;
    float v = mine_sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, v, o);
      if (l >= o) v += t;
    }
    const float prev_in_warp = __shfl_up_sync(0xffffffffu, v, 1);
    if (l == 31) wsum[w] = v;
    __syncthreads();
    if (mine_sum > 0.f) atomicMax(&last_t, tid);
    float wpre = before;
    for (int j = 0; j < w; ++j) wpre += wsum[j];
    __syncthreads();
    const float incl = wpre + v;
    const float excl = l == 0 ? wpre : wpre + prev_in_warp;
    // the last thread with mass also takes a target at or past its end (rounding)
    const bool claim = mine_sum > 0.f && excl <= target && (target < incl || tid == last_t);
    if (claim) {
      float run = excl;
      int pick = -1, lastk = -1;
      for (int i = tid; i < n; i += kThr) {
        const float e = kept_e(i);
        if (e > 0.f) {
          lastk = i;
          run += e;
          if (pick < 0 && run > target) pick = i;
        }
      }
      if (pick < 0) pick = lastk;
      const int tok = lo + pick;
      a.tok[row] = tok;
      a.lp[row] = __logf(xs[pick]) - __logf(total);
      c_arg = tok;                             // CTA 0 reads the pick for the slot update
    }
  }
  cl.sync();
  if (SLOTS && cr == 0 && tid == 0) post_update(*cl.map_shared_rank(&c_arg, owner));
  cl.sync();   // no CTA leaves while CTA 0 may still read its shared memory
}

int sample_cluster_chunk(int V) {
  const int c = (V + kCl - 1) / kCl;
  return (c + 7) / 8 * 8;
}

int sample_cluster_launch(const SampleClusterArgs& a0, bool bf16, bool slots, cudaStream_t st) {
  if (a0.R == 0) return 0;
  SampleClusterArgs a = a0;
  a.chunk = sample_cluster_chunk(a.V);
  const int smem = a.chunk * 4;
  if (smem > 200 * 1024) return -100;
  const dim3 grid(a.R * kCl), block(kThr);
#define RZ_SC(B, S)                                                                   \
  {                                                                                   \
    opt_in_smem<sample_cluster_kernel<B, S>>(smem);                                   \
    cudaFuncAttributes fa{};                                                          \
    if (cudaFuncGetAttributes(&fa, sample_cluster_kernel<B, S>) != cudaSuccess ||     \
        fa.maxDynamicSharedSizeBytes < smem)                                          \
      return -101;                                                                    \
    sample_cluster_kernel<B, S><<<grid, block, smem, st>>>(a);                        \
  }
  if (bf16 && slots) RZ_SC(true, true)
  else if (bf16) RZ_SC(true, false)
  else if (slots) RZ_SC(false, true)
  else RZ_SC(false, false)
#undef RZ_SC
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------- slot set-up
// Scatters the parameters of newly assigned slots into the tables and, for slots with
// penalties, rebuilds their prompt bitmask and output counts from the uploaded token
// lists (prompt tokens [tok_off[2i], tok_off[2i+1]), output tokens [tok_off[2i+1],
// tok_off[2i+2])).  One CTA per new slot.
__global__ void __launch_bounds__(256) sample_slot_init_kernel(SampleSlotInit u, SampleSlotTables st, int V) {
  const int i = blockIdx.x;
  const int slot = u.slot[i];
  for (int k = threadIdx.x; k < 8; k += blockDim.x) {
    st.f32[slot * 8 + k] = u.f32[i * 8 + k];
    st.i32[slot * 8 + k] = u.i32[i * 8 + k];
  }
  if (threadIdx.x == 0) {
    st.n_gen[slot] = u.n_gen[i];
    st.seed[slot] = u.seed[i];
  }
  const int nb = u.i32[i * 8 + 3], ns = u.i32[i * 8 + 4];
  for (int k = threadIdx.x; k < nb; k += blockDim.x) {
    st.bias_tok[slot * kSampMaxBias + k] = u.bias_tok[i * kSampMaxBias + k];
    st.bias_val[slot * kSampMaxBias + k] = u.bias_val[i * kSampMaxBias + k];
  }
  for (int k = threadIdx.x; k < ns; k += blockDim.x) st.stop_ids[slot * kSampMaxStop + k] = u.stop_ids[i * kSampMaxStop + k];
  const int pen = u.i32[i * 8 + 2];
  if (pen < 0) return;
  const int64_t cw = (V + 1) / 2, sw = (V + 31) / 32;
  uint32_t* cnt = st.cnt + pen * cw;
  uint32_t* seen = st.seen + pen * sw;
  for (int64_t k = threadIdx.x; k < cw; k += blockDim.x) cnt[k] = 0;
  for (int64_t k = threadIdx.x; k < sw; k += blockDim.x) seen[k] = 0;
  __syncthreads();
  const int p0 = u.tok_off[2 * i], p1 = u.tok_off[2 * i + 1], p2 = u.tok_off[2 * i + 2];
  for (int k = p0 + threadIdx.x; k < p1; k += blockDim.x) {
    const int t = u.toks[k];
    if (t >= 0 && t < V) atomicOr(&seen[t >> 5], 1u << (t & 31));
  }
  for (int k = p1 + threadIdx.x; k < p2; k += blockDim.x) {
    const int t = u.toks[k];
    if (t >= 0 && t < V) atomicAdd(&cnt[t >> 1], (t & 1) ? 0x10000u : 1u);
  }
}

int sample_slot_init_launch(const SampleSlotInit& u, int n, const SampleSlotTables& st, int V, cudaStream_t s) {
  if (n == 0) return 0;
  sample_slot_init_kernel<<<n, 256, 0, s>>>(u, st, V);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz
