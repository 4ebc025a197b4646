// Token sampling with one thread-block cluster per row of logits.
//
// The row (bf16 or fp32, up to ~400K entries) is split over the 8 CTAs of a
// cluster; each CTA reads its slice from HBM exactly once into shared memory,
// and every later pass (penalties, max, normaliser, the rejection rounds of
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
//   otherwise  e = exp((x - max) / T) = p / p_max; the kept set K holds the
//              tokens t with fewer than k tokens strictly more likely, with the
//              mass of strictly more likely tokens < top_p, and with e_t >=
//              min_p (the most likely token is always kept); one token is drawn
//              from K with probability proportional to e.
//
// K is never materialised.  The draw is exact rejection sampling with a pivot
// (no sort, no histogram): draw a candidate c from the tokens above the pivot
// in proportion to e (inverse CDF with one uniform from a counter-based
// Philox4x32-10 stream keyed by (seed, tokens generated so far, round)); one
// pass then counts the tokens and the mass strictly above e_c.  If c meets
// every rule it is in K and is returned: conditioned on acceptance it is
// distributed like e over K.  Otherwise every token at or below e_c fails too
// (the count and the mass above a token only grow as e falls), so the pivot
// rises to e_c, and the mass just computed is the next round's total.  For
// top-p at 0.9 the first candidate is accepted nine times in ten; top-k over a
// flat distribution halves the candidate set per round in expectation.  A
// round costs one pass over shared memory and two cluster barriers.
//
// The draw walks the mass in (thread, stride) order rather than token order:
// thread t of a CTA owns tokens t, t + 512, ...; per-thread sums, a total per
// cluster rank, and the uniform pick the CTA, the thread, then the token where
// the running mass crosses u times the total.  Any fixed order gives the same
// distribution.
//
// The returned logprob is that of the drawn token under the temperature-scaled
// softmax over the whole vocabulary (log e_c - log sum e), the greedy one under
// the raw softmax.
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
constexpr int kMaxRounds = 64; // rejection rounds before the most likely token is returned

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

template <bool BF16>
__device__ __forceinline__ float load1(const void* row, int64_t i) {
  if (BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(row)[i]);
  return static_cast<const float*>(row)[i];
}

}  // namespace

template <bool BF16, bool SLOTS>
__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kThr, 3) sample_cluster_kernel(SampleClusterArgs a) {
  cg::cluster_group cl = cg::this_cluster();
  const int cr = static_cast<int>(cl.block_rank());
  const int row = blockIdx.x / kCl;
  const int tid = threadIdx.x;
  extern __shared__ __align__(16) float xs[];
  __shared__ float tsum[kThr];
  __shared__ float rv[32];
  __shared__ int ri[32];
  __shared__ float wsum[kThr / 32];
  // per-CTA partial results that the other CTAs read through DSMEM (double-buffered by
  // round parity, so a round's values are never overwritten while a peer may read them)
  __shared__ float c_max, c_sum;
  __shared__ int c_arg;
  __shared__ float c_mass[2];
  __shared__ int c_cnt[2];
  __shared__ float cand_e[2];
  __shared__ int cand_t[2];
  __shared__ int last_t;

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
    tsum[tid] = z;
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

  // ---------------------------------------------------------------- 4. rejection rounds with a rising pivot
  // tsum holds each thread's mass above the pivot (initially all of it: the Z partials)
  const int k = top_k > 0 ? min(top_k, V) : V;
  const float pZ = top_p < 1.f ? top_p * Z : INFINITY;
  float ctot[kCl];
#pragma unroll
  for (int r = 0; r < kCl; ++r) ctot[r] = *cl.map_shared_rank(&c_sum, r);
  float pivot = -1.f;       // candidates: e > pivot
  float total = Z;
  int tok = arg;
  float etok = 1.f;
  for (int round = 0; round < kMaxRounds; ++round) {
    const int par = round & 1;
    // -- draw a candidate above the pivot: the CTA, then the thread, then the token
    const P4 rnd = philox10(P4{static_cast<uint32_t>(round), static_cast<uint32_t>(off),
                               static_cast<uint32_t>(off >> 32), 0x5A4D504Cu},
                            static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    const float target = unit_open(rnd.x) * total;
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
    if (owner < 0) {            // rounding past the end: the last CTA with mass
      owner = last < 0 ? 0 : last;
      before = acc - (last < 0 ? 0.f : ctot[last]);
    }
    if (cr == owner) {
      // inclusive prefix of the per-thread sums in thread order; thread i owns
      // [P(i-1), P(i)), with P(i-1) taken from its neighbour so ranges neither overlap nor gap
      const int w = tid >> 5, l = tid & 31;
      const float mine = tsum[tid];
      float v = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, v, o);
        if (l >= o) v += t;
      }
      const float prev = __shfl_up_sync(0xffffffffu, v, 1);
      if (l == 31) wsum[w] = v;
      if (tid == 0) {
        cand_t[par] = arg;      // replaced below; kept if rounding leaves no claimant
        cand_e[par] = 1.f;
        last_t = -1;
      }
      __syncthreads();
      float wpre = before;
      for (int j = 0; j < w; ++j) wpre += wsum[j];
      if (mine > 0.f) atomicMax(&last_t, tid);   // the last thread with mass also takes a target past its end
      __syncthreads();
      const float incl = wpre + v;
      const float excl = l == 0 ? wpre : wpre + prev;
      if (mine > 0.f && excl <= target && (target < incl || tid == last_t)) {
        float run = excl;
        int pick = -1, lastk = -1;
        for (int i = tid; i < n; i += kThr) {
          const float e = xs[i];
          if (e > pivot) {
            lastk = i;
            run += e;
            if (pick < 0 && run > target) pick = i;
          }
        }
        if (pick < 0) pick = lastk;
        if (pick >= 0) {
          cand_t[par] = lo + pick;
          cand_e[par] = xs[pick];
        }
      }
    }
    cl.sync();
    const int c = *cl.map_shared_rank(&cand_t[par], owner);
    const float ec = *cl.map_shared_rank(&cand_e[par], owner);
    // -- count and mass strictly above the candidate (the next round's sums if it fails)
    float ms = 0.f;
    int cn = 0;
    for (int i = tid; i < n; i += kThr) {
      const float e = xs[i];
      if (e > ec) {
        ms += e;
        ++cn;
      }
    }
    tsum[tid] = ms;
    const float cms = block_sum(ms, rv);
    const int ccn = static_cast<int>(block_sum(static_cast<float>(cn), rv));
    if (tid == 0) {
      c_mass[par] = cms;
      c_cnt[par] = ccn;
    }
    cl.sync();
    float above = 0.f;
    long nabove = 0;
#pragma unroll
    for (int r = 0; r < kCl; ++r) {
      ctot[r] = *cl.map_shared_rank(&c_mass[par], r);
      above += ctot[r];
      nabove += *cl.map_shared_rank(&c_cnt[par], r);
    }
    tok = c;
    etok = ec;
    // (the most likely token, e = 1, has nothing above it and always passes)
    if ((nabove < k && above < pZ && ec >= min_p) || ec >= 1.f) break;
    if (!(above > 0.f)) {       // nothing left above the candidate: the most likely token
      tok = arg;
      etok = 1.f;
      break;
    }
    pivot = ec;
    total = above;
    if (round == kMaxRounds - 1) {
      tok = arg;
      etok = 1.f;
    }
  }
  if (cr == 0 && tid == 0) {
    a.tok[row] = tok;
    a.lp[row] = __logf(etok) - __logf(Z);
    post_update(tok);
  }
  cl.sync();   // no CTA leaves while a peer may still read its shared memory
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
