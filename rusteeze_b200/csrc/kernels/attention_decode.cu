// Paged-KV decode attention (one query token per sequence), split-KV.
//
// The reference has no working decode path: its paged cache read returns
// zeros (crates/rusteeze-tensor/src/cache.rs:508-527) and its models use a
// contiguous per-sequence cache with materialised QK^T (crates/rusteeze-
// model/src/architectures/common.rs:262-293).  Math here follows the online
// softmax of its CPU FlashAttention (crates/rusteeze-engine/src/
// flash_attention.rs:186-252).
//
// Grid (splits, Hkv, seqs); 128 threads.  A CTA owns one (sequence, kv head,
// KV range) and all G = Hq/Hkv query heads of that kv head, so each KV byte
// is read from HBM once.  Cache layout per layer: [blocks, Hkv, 16, D] with
// a runtime block stride, so every (block, head) page is one contiguous
// 16*D*2-byte run that a single 1-D bulk copy (cp.async.bulk) moves into a
// 4-stage shared-memory ring, two pages (32 tokens) per stage.
//   scores : 4 threads per token, each a quarter of D (rotated 16-byte
//            chunks: bank-conflict free), reduced with 2 shuffles
//   softmax: online max/sum per head, one warp per head
//   PV     : thread = (token half, dim pair); halves merged at the end
// With splits > 1 each CTA writes (acc, max, sum) partials to a workspace
// and `decode_combine` merges them; the split count is fixed per launch and
// each CTA derives its KV range from the live sequence length, so one
// CUDA graph serves any context length.
#include "attention.h"
#include "common.cuh"

namespace rz {

constexpr int kDecThreads = 128;
constexpr int kPagesPerStage = 2;
constexpr int kTokPerStage = 16 * kPagesPerStage;
constexpr int kDecStages = 4;

template <int D, int G>
struct DecSmem {
  static constexpr int kPageBytes = 16 * D * 2;
  static constexpr int kStageBytes = 2 * kPagesPerStage * kPageBytes;  // K and V
  static constexpr int kBytes = kDecStages * kStageBytes + G * D * 4 /*q*/ + G * kTokPerStage * 4 /*scores*/ +
                                4 * G * 4 /*stats*/ + 64 /*bars*/ + 2 * G * D * 4 /*PV merge*/ + 128;
};

template <int D, int G>
__global__ void __launch_bounds__(kDecThreads)
    decode_attn_kernel(DecodeAttnParams p) {
  using SM = DecSmem<D, G>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  float* q_s = reinterpret_cast<float*>(smem + kDecStages * SM::kStageBytes);
  float* sc = q_s + G * D;                    // [G][32]
  float* corr = sc + G * kTokPerStage;        // [G] rescale factors of this stage
  float* lsum = corr + G;                     // [G] running sums
  float* mrun = lsum + G;                     // [G] running maxima
  uint64_t* bars = reinterpret_cast<uint64_t*>(mrun + G + (G & 1));
  float* merge = reinterpret_cast<float*>(bars + kDecStages);

  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int L = p.seq_lens[seq];
  if (L < 0 || L > p.bt_stride * 16) {  // longer than its block-table row: record, clamp
    set_status(p.status, kBadArgument);
    L = L < 0 ? 0 : static_cast<int>(p.bt_stride * 16);
  }
  const int nblk = (L + 15) >> 4;
  const int per = (nblk + p.num_splits - 1) / p.num_splits;
  const int b0 = split * per;
  const int b1 = min(nblk, b0 + per);
  const int nstage = b1 > b0 ? (b1 - b0 + kPagesPerStage - 1) / kPagesPerStage : 0;
  const int32_t* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride;

  // q (pre-scaled) -> smem fp32
  for (int i = tid; i < G * D; i += kDecThreads) {
    const int g = i / D, d = i % D;
    q_s[i] = bf2f(p.q[static_cast<int64_t>(seq) * p.q_stride + (kvh * G + g) * D + d]) * p.scale;
  }
  if (tid < G) {
    lsum[tid] = 0.f;
    mrun[tid] = -INFINITY;
  }
  if (tid == 0) {
    for (int s = 0; s < kDecStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int st) {
    // thread 0: bulk-copy up to kPagesPerStage K and V pages of stage `st` into ring slot st % kDecStages
    uint8_t* slot = ring + (st % kDecStages) * SM::kStageBytes;
    const int blo = b0 + st * kPagesPerStage;
    const int np = min(kPagesPerStage, b1 - blo);
    mbar_arrive_expect_tx(&bars[st % kDecStages], 2 * np * SM::kPageBytes);
    for (int j = 0; j < np; ++j) {
      int64_t page = bt[blo + j];
      if (page < 0 || page >= p.num_blocks) {  // corrupt block table: record and read page 0 instead
        set_status(p.status, kBadArgument);
        page = 0;
      }
      const __nv_bfloat16* ksrc = p.k_cache + page * p.block_stride + static_cast<int64_t>(kvh) * 16 * D;
      const __nv_bfloat16* vsrc = p.v_cache + page * p.block_stride + static_cast<int64_t>(kvh) * 16 * D;
      bulk_load(slot + j * SM::kPageBytes, ksrc, SM::kPageBytes, &bars[st % kDecStages]);
      bulk_load(slot + (kPagesPerStage + j) * SM::kPageBytes, vsrc, SM::kPageBytes, &bars[st % kDecStages]);
    }
  };
  if (tid == 0)
    for (int s = 0; s < kDecStages && s < nstage; ++s) issue(s);

  // PV roles: thread = (token half th, dim pair dp)
  constexpr int kPairs = D / 2;
  constexpr int kPvThreads = 2 * kPairs;     // D=128 -> 128 threads
  constexpr int kDimIters = (kPvThreads + kDecThreads - 1) / kDecThreads;
  float acc[kDimIters][G][2];
#pragma unroll
  for (int a = 0; a < kDimIters; ++a)
#pragma unroll
    for (int g = 0; g < G; ++g) acc[a][g][0] = acc[a][g][1] = 0.f;
  bool ok = true;
  const int kv_end = min(L, b1 * 16);         // keys this CTA owns: [b0*16, kv_end)

  for (int st = 0; st < nstage; ++st) {
    if (ok && !mbar_wait(&bars[st % kDecStages], (st / kDecStages) & 1, p.status, kAttnTimeout)) ok = false;
    const uint8_t* slot = ring + (st % kDecStages) * SM::kStageBytes;
    const __nv_bfloat16* Ks = reinterpret_cast<const __nv_bfloat16*>(slot);
    const __nv_bfloat16* Vs = reinterpret_cast<const __nv_bfloat16*>(slot + kPagesPerStage * SM::kPageBytes);
    const int tok0 = (b0 + st * kPagesPerStage) * 16;
    // ---- scores: token t = tid/4, quarter qd = tid%4
    {
      const int t = tid >> 2, qd = tid & 3;
      constexpr int kChunks = D / 8;          // 16-byte chunks per row
      constexpr int kMine = kChunks / 4;      // chunks per thread
      float part[G];
#pragma unroll
      for (int g = 0; g < G; ++g) part[g] = 0.f;
#pragma unroll
      for (int i = 0; i < kMine; ++i) {
        const int c = qd + 4 * ((i + t) % kMine);
        uint4 u = *reinterpret_cast<const uint4*>(Ks + t * D + c * 8);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f = __bfloat1622float2(h[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4* qv = reinterpret_cast<const float4*>(q_s + g * D + c * 8);
          const float4 q0 = qv[0], q1 = qv[1];
          part[g] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] + q1.y * kf[5] +
                     q1.z * kf[6] + q1.w * kf[7];
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        part[g] += __shfl_xor_sync(0xffffffffu, part[g], 1);
        part[g] += __shfl_xor_sync(0xffffffffu, part[g], 2);
      }
      if (qd == 0) {
        const int pos = tok0 + t;
        const bool valid = pos < kv_end && (p.window <= 0 || pos > L - 1 - p.window);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float s = part[g];
          if (p.softcap > 0.f) s = p.softcap * tanhf(s / p.softcap);
          sc[g * kTokPerStage + t] = valid ? s : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax: warp w handles heads w, w+4, ...
    for (int g = warp; g < G; g += kDecThreads / 32) {
      const float s = sc[g * kTokPerStage + lane];
      const float mx = warp_max(s);
      const float m_old = mrun[g];
      const float m_new = fmaxf(m_old, mx);
      const float pr = m_new == -INFINITY ? 0.f : __expf(s - m_new);
      const float sum = warp_sum(pr);
      sc[g * kTokPerStage + lane] = pr;
      __syncwarp();
      if (lane == 0) {
        const float cf = m_old == -INFINITY ? 0.f : __expf(m_old - m_new);
        corr[g] = cf;
        lsum[g] = lsum[g] * cf + sum;
        mrun[g] = m_new;
      }
    }
    __syncthreads();
    // ---- PV (only over tokens of this stage that hold data: stale ring bytes may be NaN)
    const int ntok = min(kTokPerStage, kv_end - tok0);
#pragma unroll
    for (int a = 0; a < kDimIters; ++a) {
      const int idx = tid + a * kDecThreads;
      if (idx < kPvThreads) {
        const int th = idx / kPairs, dp = idx % kPairs;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          acc[a][g][0] *= corr[g];
          acc[a][g][1] *= corr[g];
        }
        const int t_end = min(th * 16 + 16, ntok);
#pragma unroll 4
        for (int t = th * 16; t < t_end; ++t) {
          const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(Vs + t * D + 2 * dp));
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float pr = sc[g * kTokPerStage + t];
            acc[a][g][0] += pr * v.x;
            acc[a][g][1] += pr * v.y;
          }
        }
      }
    }
    __syncthreads();  // ring slot and scores free
    if (tid == 0 && ok && st + kDecStages < nstage) issue(st + kDecStages);
  }

  // ---- merge the two token halves, then normalise / emit partials
#pragma unroll
  for (int a = 0; a < kDimIters; ++a) {
    const int idx = tid + a * kDecThreads;
    if (idx < kPvThreads && idx >= kPairs) {
      const int dp = idx - kPairs;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        merge[(g * D) + 2 * dp] = acc[a][g][0];
        merge[(g * D) + 2 * dp + 1] = acc[a][g][1];
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int a = 0; a < kDimIters; ++a) {
    const int idx = tid + a * kDecThreads;
    if (idx < kPairs) {
      const int dp = idx;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float o0 = acc[a][g][0] + merge[g * D + 2 * dp];
        const float o1 = acc[a][g][1] + merge[g * D + 2 * dp + 1];
        const int qh = kvh * G + g;
        if (p.num_splits == 1) {
          const float l = lsum[g];
          const float inv = l > 0.f ? 1.f / l : 0.f;
          __nv_bfloat162 r = __floats2bfloat162_rn(o0 * inv, o1 * inv);
          *reinterpret_cast<__nv_bfloat162*>(p.out + static_cast<int64_t>(seq) * p.out_stride + qh * D + 2 * dp) = r;
        } else {
          float* w = p.workspace + ((static_cast<int64_t>(seq) * p.num_q_heads + qh) * p.num_splits + split) * (D + 2);
          w[2 * dp] = o0;
          w[2 * dp + 1] = o1;
          if (dp == 0) {
            w[D] = mrun[g];
            w[D + 1] = lsum[g];
          }
        }
      }
    }
  }
}

template <int D>
__global__ void decode_combine_kernel(DecodeAttnParams p) {
  const int qh = blockIdx.x, seq = blockIdx.y;
  const float* w = p.workspace + (static_cast<int64_t>(seq) * p.num_q_heads + qh) * p.num_splits * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.num_splits; ++s) M = fmaxf(M, w[s * (D + 2) + D]);
  float den = 0.f;
  for (int s = 0; s < p.num_splits; ++s) {
    const float m = w[s * (D + 2) + D];
    den += m == -INFINITY ? 0.f : __expf(m - M) * w[s * (D + 2) + D + 1];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    for (int s = 0; s < p.num_splits; ++s) {
      const float m = w[s * (D + 2) + D];
      if (m != -INFINITY) o += __expf(m - M) * w[s * (D + 2) + d];
    }
    p.out[static_cast<int64_t>(seq) * p.out_stride + qh * D + d] = f2bf(o * inv);
  }
}

template <int D, int G>
static int launch_dec(const DecodeAttnParams& p, cudaStream_t st) {
  using SM = DecSmem<D, G>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(decode_attn_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM::kBytes);
    attr = true;
  }
  dim3 grid(p.num_splits, p.num_kv_heads, p.num_seqs);
  decode_attn_kernel<D, G><<<grid, kDecThreads, SM::kBytes, st>>>(p);
  if (p.num_splits > 1) decode_combine_kernel<D><<<dim3(p.num_q_heads, p.num_seqs), 128, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int decode_attention_launch(const DecodeAttnParams& p, cudaStream_t st) {
  if (p.num_seqs == 0) return 0;
  const int G = p.num_q_heads / p.num_kv_heads;
#define RZ_DEC(DD, GG) \
  if (p.head_dim == DD && G == GG) return launch_dec<DD, GG>(p, st);
  RZ_DEC(128, 1) RZ_DEC(128, 2) RZ_DEC(128, 4) RZ_DEC(128, 8)
  RZ_DEC(64, 1) RZ_DEC(64, 2) RZ_DEC(64, 4) RZ_DEC(64, 8)
  RZ_DEC(256, 1) RZ_DEC(256, 2) RZ_DEC(256, 4) RZ_DEC(256, 8)
#undef RZ_DEC
  return -100;  // unsupported (head_dim, group) combination: caller splits heads
}

}  // namespace rz
