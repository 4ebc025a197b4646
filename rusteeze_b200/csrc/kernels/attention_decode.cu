// Paged-KV decode attention (one query token per sequence), split-KV.
//
// The reference has no working decode path: its paged cache read returns
// zeros (crates/rusteeze-tensor/src/cache.rs:508-527) and its models use a
// contiguous per-sequence cache with materialised QK^T (crates/rusteeze-
// model/src/architectures/common.rs:262-293).  Math here follows the online
// softmax of its CPU FlashAttention (crates/rusteeze-engine/src/
// flash_attention.rs:186-252).
//
// Work item = (sequence, kv head, KV split).  Each WARP owns one item and
// runs independently -- no CTA-wide barrier in the loop:
//   * the G = Hq/Hkv query heads of the kv head are packed into the M
//     dimension of a 16-row tensor-core tile (rows >= G are zero), so
//     S = Q K^T and O += P V are mma.sync m16n8k16 (bf16 in, fp32 acc) and
//     every KV byte is read from HBM once for all G heads;
//   * pages (16 tokens; K and V each one contiguous 16*D*2-byte run in the
//     [blocks, Hkv, 16, D] per-layer cache view) stream into a per-warp
//     shared-memory ring with cp.async, XOR-swizzled so ldmatrix is
//     bank-conflict free; the warp keeps kStages pages in flight;
//   * online softmax per head in registers (2 shuffles per row max/sum).
// With splits > 1 each item writes (acc, max, sum) partials to a workspace
// and `decode_combine` merges them.  The split count is fixed per launch;
// each item derives its page range from the live sequence length, so one
// CUDA graph serves any context length.
#include "attention.h"
#include "common.cuh"

namespace rz {


__device__ __forceinline__ void dec_cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void dec_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void dec_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void dec_ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void dec_ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
__device__ __forceinline__ void dec_mma(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void dec_mma_h(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t dec_pack(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t dec_pack_h(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// fp8 cache pages: the tensor cores take f16 operands here (the fp8 value sets of e4m3 and
// e5m2 are exactly representable in f16), so K/V pages, Q and P are f16 for these variants
template <int KVF>
__device__ __forceinline__ void mma_kv(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  if constexpr (KVF == kKvBf16) dec_mma(c, a0, a1, a2, a3, b0, b1);
  else dec_mma_h(c, a0, a1, a2, a3, b0, b1);
}
template <int KVF>
__device__ __forceinline__ uint32_t pack_kv(float a, float b) {
  if constexpr (KVF == kKvBf16) return dec_pack(a, b);
  else return dec_pack_h(a, b);
}
// two fp8 values (low byte first) -> f16x2 (first value in the low half)
template <int KVF>
__device__ __forceinline__ uint32_t fp8x2_to_h2(uint32_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xffffu),
                                                   KVF == kKvE4m3 ? __NV_E4M3 : __NV_E5M2);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}

template <int D, int KVF>
struct DecCfg {
  static constexpr bool kF8 = KVF != kKvBf16;
  static constexpr int kWarps = D <= 128 ? 8 : 4;
  static constexpr int kPage = 16 * D * 2;                      // bytes of one 16-bit K (or V) page
  static constexpr int kRingPage = kF8 ? 16 * D : kPage;        // bytes of one page as the cache holds it
  static constexpr int kStages = kF8 ? (D <= 64 ? 8 : (D <= 128 ? 4 : 3)) : (D <= 64 ? 6 : (D <= 128 ? 3 : 2));
  static constexpr int kConvBytes = kF8 ? 2 * kPage : 0;        // f16 K and V page converted from the ring
  static constexpr int kWarpBytes = kStages * 2 * kRingPage + kConvBytes + 16 * D * 2;  // ring + conv + Q tile
  static constexpr int kSmem = kWarps * kWarpBytes;
  static_assert(kSmem <= 227 * 1024, "decode attention shared memory");
};

// (row, 16-byte chunk) -> byte offset inside a [16][D] bf16 page/tile, XOR swizzled
template <int D>
__device__ __forceinline__ uint32_t dswz(int row, int chunk) {
  return static_cast<uint32_t>(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

template <int D, bool ALIBI, int KVF>
__global__ void __launch_bounds__(DecCfg<D, KVF>::kWarps * 32, 1) decode_attn_kernel(DecodeAttnParams p) {
  using C = DecCfg<D, KVF>;
  constexpr int kChunks = D / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* wbase = smem + warp * C::kWarpBytes;
  const uint32_t aRing = smem_u32(wbase);
  uint8_t* sConv = wbase + C::kStages * 2 * C::kRingPage;       // fp8 variants only
  const uint32_t aConv = aRing + C::kStages * 2 * C::kRingPage;
  const uint32_t aQ = aConv + C::kConvBytes;
  uint8_t* sQ = sConv + C::kConvBytes;

  const int item = blockIdx.x * C::kWarps + warp;
  const int n_items = p.num_seqs * p.num_kv_heads * p.num_splits;
  if (item >= n_items) return;
  const int split = item % p.num_splits;
  const int kvh = (item / p.num_splits) % p.num_kv_heads;
  const int seq = item / (p.num_splits * p.num_kv_heads);
  const int G = p.num_q_heads / p.num_kv_heads;

  int L = p.seq_lens[seq];
  if (L < 0 || L > p.bt_stride * 16) {  // longer than its block-table row: record, clamp
    set_status(p.status, kBadArgument);
    L = L < 0 ? 0 : static_cast<int>(p.bt_stride * 16);
  }
  const int nblk = (L + 15) >> 4;
  const int per = (nblk + p.num_splits - 1) / p.num_splits;
  const int b0 = split * per;
  const int b1 = min(nblk, b0 + per);
  const int npages = b1 > b0 ? b1 - b0 : 0;
  const int32_t* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride;

  // Q tile: rows g < G are the query heads of this kv head, rows >= G are zero (f16 for
  // the fp8-cache variants)
  for (int i = lane; i < 16 * kChunks; i += 32) {
    const int r = i / kChunks, c = i % kChunks;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G)
      v = *reinterpret_cast<const uint4*>(p.q + static_cast<int64_t>(seq) * p.q_stride +
                                          static_cast<int64_t>(kvh * G + r) * D + c * 8);
    if constexpr (C::kF8) {
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
      uint32_t h[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(b[k]);
        h[k] = dec_pack_h(f.x, f.y);
      }
      v = make_uint4(h[0], h[1], h[2], h[3]);
    }
    *reinterpret_cast<uint4*>(sQ + dswz<D>(r, c)) = v;
  }

  auto load_page = [&](int j, int slot) {
    int64_t pid = bt[b0 + j];
    if (pid < 0 || pid >= p.num_blocks) {  // corrupt block table: record and read page 0 instead
      set_status(p.status, kBadArgument);
      pid = 0;
    }
    const int64_t off = pid * p.block_stride + static_cast<int64_t>(kvh) * 16 * D;
    const uint32_t dk = aRing + slot * 2 * C::kRingPage;
    const uint32_t dv = dk + C::kRingPage;
    if constexpr (C::kF8) {
      // a page is 16 * D contiguous bytes: 16-byte pieces in order (converted after landing)
      const uint8_t* gk = reinterpret_cast<const uint8_t*>(p.k_cache) + off;
      const uint8_t* gv = reinterpret_cast<const uint8_t*>(p.v_cache) + off;
#pragma unroll
      for (int i = lane; i < D; i += 32) {
        dec_cp_async16(dk + i * 16, gk + i * 16);
        dec_cp_async16(dv + i * 16, gv + i * 16);
      }
    } else {
#pragma unroll
      for (int i = lane; i < 16 * kChunks; i += 32) {
        const int r = i / kChunks, c = i % kChunks;
        dec_cp_async16(dk + dswz<D>(r, c), p.k_cache + off + r * D + c * 8);
        dec_cp_async16(dv + dswz<D>(r, c), p.v_cache + off + r * D + c * 8);
      }
    }
  };
  // prologue: kStages-1 pages in flight (empty groups keep the group count uniform)
#pragma unroll
  for (int s = 0; s < C::kStages - 1; ++s) {
    if (s < npages) load_page(s, s);
    dec_commit();
  }
  __syncwarp();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  // fp8 cache: K holds k / k_scale, so the logit scale takes k_scale; V's scale goes on O
  const float qk_scale = C::kF8 ? p.scale * p.k_scale : p.scale;
  const float v_scale = C::kF8 ? p.v_scale : 1.f;
  const float sl2 = qk_scale * 1.4426950408889634f;
  // ALiBi slope of the thread's two head rows (lane/4, lane/4 + 8), log2 domain
  float ab[2] = {0.f, 0.f};
  if (ALIBI) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = (lane >> 2) + 8 * h;
      ab[h] = r < G ? p.alibi[kvh * G + r] * 1.4426950408889634f : 0.f;
    }
  }
  const int kv_end = min(L, b1 * 16);

  for (int j = 0; j < npages; ++j) {
    const int nxt = j + C::kStages - 1;
    if (nxt < npages) load_page(nxt, nxt % C::kStages);
    dec_commit();
    dec_wait<C::kStages - 1>();
    __syncwarp();
    uint32_t aK = aRing + (j % C::kStages) * 2 * C::kPage;
    if constexpr (C::kF8) {
      // fp8 K and V page (ring slot j % kStages) -> swizzled f16 page in sConv
      const uint8_t* src = wbase + (j % C::kStages) * 2 * C::kRingPage;
#pragma unroll 4
      for (int i = lane; i < 2 * 16 * kChunks; i += 32) {
        const int kv = i / (16 * kChunks), rem = i % (16 * kChunks);
        const int r = rem / kChunks, c = rem % kChunks;
        const uint2 raw = *reinterpret_cast<const uint2*>(src + kv * C::kRingPage + r * D + c * 8);
        *reinterpret_cast<uint4*>(sConv + kv * C::kPage + dswz<D>(r, c)) =
            make_uint4(fp8x2_to_h2<KVF>(raw.x), fp8x2_to_h2<KVF>(raw.x >> 16), fp8x2_to_h2<KVF>(raw.y),
                       fp8x2_to_h2<KVF>(raw.y >> 16));
      }
      __syncwarp();
      aK = aConv;
    }
    const uint32_t aV = aK + C::kPage;
    // ---- S[16 heads x 16 tokens]
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3, b0r, b1r, b2r, b3r;
      dec_ldsm_x4(aQ + dswz<D>(lane & 15, 2 * kk + (lane >> 4)), a0, a1, a2, a3);
      dec_ldsm_x4(aK + dswz<D>((lane & 7) + ((lane >> 4) << 3), 2 * kk + ((lane >> 3) & 1)), b0r, b1r, b2r, b3r);
      mma_kv<KVF>(s[0], a0, a1, a2, a3, b0r, b1r);
      mma_kv<KVF>(s[1], a0, a1, a2, a3, b2r, b3r);
    }
    // ---- mask + online softmax (log2 domain); thread rows: lane/4 and lane/4 + 8
    const int tok0 = (b0 + j) * 16;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int pos = tok0 + nt * 8 + 2 * (lane & 3) + (e & 1);
        float v = s[nt][e];
        if (p.softcap > 0.f) v = p.softcap * tanhf(v * qk_scale / p.softcap) * 1.4426950408889634f;
        else v *= sl2;
        if (ALIBI) v += ab[e >> 1] * static_cast<float>(pos - (L - 1));
        const bool valid = pos < kv_end && (p.window <= 0 || pos > L - 1 - p.window);
        v = valid ? v : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float mn = fmaxf(m_r[h], mx[h]);
      corr[h] = (m_r[h] == -INFINITY) ? 0.f : exp2f(m_r[h] - mn);
      m_r[h] = mn;
      l_r[h] *= corr[h];
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float pv = m_r[h] == -INFINITY ? 0.f : exp2f(s[nt][e] - m_r[h]);
        s[nt][e] = pv;
        l_r[h] += pv;
      }
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    // ---- O += P V   (P: 16 heads x 16 tokens as the A operand)
    const uint32_t pa0 = pack_kv<KVF>(s[0][0], s[0][1]), pa1 = pack_kv<KVF>(s[0][2], s[0][3]);
    const uint32_t pa2 = pack_kv<KVF>(s[1][0], s[1][1]), pa3 = pack_kv<KVF>(s[1][2], s[1][3]);
#pragma unroll
    for (int dn = 0; dn < D / 16; ++dn) {
      uint32_t b0r, b1r, b2r, b3r;
      dec_ldsm_x4_t(aV + dswz<D>((lane & 7) + (((lane >> 3) & 1) << 3), 2 * dn + (lane >> 4)), b0r, b1r, b2r, b3r);
      mma_kv<KVF>(o[2 * dn], pa0, pa1, pa2, pa3, b0r, b1r);
      mma_kv<KVF>(o[2 * dn + 1], pa0, pa1, pa2, pa3, b2r, b3r);
    }
    __syncwarp();  // ring slot j % kStages is refilled next iteration
  }
  dec_wait<0>();

  // ---- finalise rows g < G
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int g = (lane >> 2) + h * 8;
    if (g >= G) continue;
    const int qh = kvh * G + g;
    if (p.num_splits == 1) {
      const float inv = l_r[h] > 0.f ? v_scale / l_r[h] : 0.f;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(seq) * p.out_stride + static_cast<int64_t>(qh) * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<__nv_bfloat162*>(dst + i * 8 + 2 * (lane & 3)) =
            __floats2bfloat162_rn(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
    } else {
      float* w = p.workspace + ((static_cast<int64_t>(seq) * p.num_q_heads + qh) * p.num_splits + split) * (D + 2);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        w[i * 8 + 2 * (lane & 3)] = o[i][2 * h] * v_scale;
        w[i * 8 + 2 * (lane & 3) + 1] = o[i][2 * h + 1] * v_scale;
      }
      if ((lane & 3) == 0) {
        // running max is in log2 units; the combine kernel works in the same units
        w[D] = m_r[h];
        w[D + 1] = l_r[h];
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
    den += m == -INFINITY ? 0.f : exp2f(m - M) * w[s * (D + 2) + D + 1];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    for (int s = 0; s < p.num_splits; ++s) {
      const float m = w[s * (D + 2) + D];
      if (m != -INFINITY) o += exp2f(m - M) * w[s * (D + 2) + d];
    }
    p.out[static_cast<int64_t>(seq) * p.out_stride + qh * D + d] = f2bf(o * inv);
  }
}

template <int D, bool ALIBI, int KVF>
static void launch_dec_main(const DecodeAttnParams& p, cudaStream_t st) {
  using C = DecCfg<D, KVF>;
  opt_in_smem<decode_attn_kernel<D, ALIBI, KVF>>(C::kSmem);
  const int items = p.num_seqs * p.num_kv_heads * p.num_splits;
  decode_attn_kernel<D, ALIBI, KVF><<<(items + C::kWarps - 1) / C::kWarps, C::kWarps * 32, C::kSmem, st>>>(p);
}

template <int D, int KVF>
static void launch_dec_fmt(const DecodeAttnParams& p, cudaStream_t st) {
  if (p.alibi != nullptr) launch_dec_main<D, true, KVF>(p, st);
  else launch_dec_main<D, false, KVF>(p, st);
}

template <int D>
static int launch_dec(const DecodeAttnParams& p, cudaStream_t st) {
  if (p.kv_fmt == kKvE4m3) launch_dec_fmt<D, kKvE4m3>(p, st);
  else if (p.kv_fmt == kKvE5m2) launch_dec_fmt<D, kKvE5m2>(p, st);
  else launch_dec_fmt<D, kKvBf16>(p, st);
  if (p.num_splits > 1) decode_combine_kernel<D><<<dim3(p.num_q_heads, p.num_seqs), 128, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int decode_attention_launch(const DecodeAttnParams& p, cudaStream_t st) {
  if (p.num_seqs == 0) return 0;
  const int G = p.num_q_heads / p.num_kv_heads;
  if (G < 1 || G > 16 || p.num_q_heads % p.num_kv_heads) return -100;
  if (p.kv_fmt < kKvBf16 || p.kv_fmt > kKvE5m2) return -100;
  switch (p.head_dim) {
    case 64: return launch_dec<64>(p, st);
    case 128: return launch_dec<128>(p, st);
    case 256: return launch_dec<256>(p, st);
    default: return -100;
  }
}

}  // namespace rz
