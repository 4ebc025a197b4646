// Prefill (and chunked-prefill / multi-token verify) attention on 5th-generation
// tensor cores, for head_dim 128: FlashAttention-style online softmax with
// both GEMMs (S = Q K^T and O += P V) issued as tcgen05.mma into TMEM.
//
// One CTA per (sequence, query tile, kv head); the 128 MMA rows are the
// query tile's 128/G tokens x the G query heads sharing the kv head (GQA
// packing), so every K/V page is loaded once for the whole head group.
//
//   warp 0      TMA producer: K and V tiles of 128 positions straight from the
//               paged cache through a 4-D tensor map (d, slot, head, block):
//               8 pages x 2 swizzle halves per tile, 2-stage ring;
//   warp 1      MMA issuer: S_{j+1} = Q K_{j+1}^T is issued before O += P_j V_j
//               so the tensor core works while softmax runs on S_j;
//               S is double-buffered in TMEM (cols 0-255), O lives in 256-383;
//   warps 2..5  softmax / correction / epilogue, one query row per thread:
//               tcgen05.ld the S row, causal / sliding-window / soft-cap masks
//               in registers, exp2 online softmax with the running maximum
//               updated only when it grows by more than 2^8 (then O is
//               rescaled in TMEM with tcgen05.ld/st), P written as bf16 pairs
//               back into the thread's own S columns in TMEM (tcgen05.st), from
//               where the PV MMA takes its A operand: softmax of tile j+1 runs
//               while PV_j reads P_j, and waits for PV_j only to rescale O;
//               finally O / l -> bf16 rows.
// V stays in its natural [position][d] layout and is consumed as an MN-major
// B operand, so no transpose is needed.  Every wait is bounded; page ids
// outside the cache are recorded in the status word and page 0 is read.
#include <cudaTypedefs.h>

#include "attention.h"
#include "common.cuh"

namespace rz {

namespace {

constexpr int kTile = 16 * 1024;        // one 128-row x 128-byte swizzled half tile
constexpr int kPfThreads = 320;   // producer, MMA, 8 softmax warps (2 per TMEM lane quarter)
constexpr int kPfSmem = 10 * kTile + 1024 + 256 + 3072;   // Q(2) K(2x2) V(2x2) halves, barriers, exchange

}  // namespace

struct PfTcArgs {
  PrefillAttnParams p;
  int G;              // query heads per kv head
  int tq;             // tokens per query tile (128 / G)
  int tiles_per_seq;
};

template <bool SOFTCAP, bool WINDOW, bool ALIBI>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const PfTcArgs a) {
  const PrefillAttnParams& p = a.p;
  constexpr int D = 128;
  const int seq = p.seq_offset + blockIdx.x / a.tiles_per_seq;
  const int tile = blockIdx.x % a.tiles_per_seq;
  const int kvh = blockIdx.y;
  const int q0 = p.query_start_loc[seq];
  const int n_new = p.query_start_loc[seq + 1] - q0;
  const int tok0 = tile * a.tq;
  if (tok0 >= n_new) return;                      // uniform: nothing to do for this tile
  const int L = p.seq_lens[seq];
  const int ctx = L - n_new;
  const int ntok = min(a.tq, n_new - tok0);
  const int pos_lo = ctx + tok0, pos_hi = ctx + tok0 + ntok - 1;
  const int kv_end = pos_hi + 1;
  int kv_beg = p.window > 0 ? max(0, pos_lo - p.window + 1) : 0;
  kv_beg &= ~127;
  const int ntiles = (kv_end - kv_beg + 127) / 128;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t* sQ = smem;                    // 2 halves (d 0-63, 64-127)
  uint8_t* sK = smem + 2 * kTile;        // [stage][half]
  uint8_t* sV = smem + 6 * kTile;        // [stage][d half]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 10 * kTile);
  uint64_t* k_full = bars;               // [2]
  uint64_t* v_full = bars + 2;           // [2]
  uint64_t* kv_empty = bars + 4;         // [2]
  uint64_t* s_full = bars + 6;           // [2]
  uint64_t* s_empty = bars + 8;          // [2] S/P slot free again (PV of its tile completed)
  uint64_t* p_full = bars + 10;          // [2] P of the slot's tile stored in TMEM
  uint64_t* pv_done = bars + 16;         // the last issued PV completed (O may be rescaled)
  uint64_t* o_full = bars + 12;
  uint64_t* mx_bar = bars + 13;          // the two threads of a row exchange their half-row maxima
  uint64_t* fin_bar = bars + 14;         // ... and their half-row sums at the end
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  float* xch = reinterpret_cast<float*>(bars + 17);   // maxima [2 tile parities][2 halves][128 rows]
  float* xsum = xch + 512;                              // sums [2 halves][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 1);
      mbar_init(&p_full[i], 256);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_full, 1);
    mbar_init(mx_bar, 256);
    mbar_init(fin_bar, 256);
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);

  // Q tile -> shared memory (128-byte swizzle, K-major), all threads
  for (int i = threadIdx.x; i < 128 * 16; i += kPfThreads) {
    const int r = i >> 4, c = i & 15;
    const int t = r / a.G, g = r % a.G;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < ntok)
      v = *reinterpret_cast<const uint4*>(p.q + static_cast<size_t>(q0 + tok0 + t) * p.q_stride +
                                          (kvh * a.G + g) * D + c * 8);
    const int half = c >> 3, cc = c & 7;
    *reinterpret_cast<uint4*>(sQ + half * kTile + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int32_t* bt = p.block_tables + static_cast<size_t>(seq) * p.bt_stride;
      const int last_page = (L - 1) / 16;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1, u = j >> 1;
        if (u >= 1 && !mbar_wait(&kv_empty[s], (u - 1) & 1, p.status, kAttnTimeout)) break;
        int blk[8];
#pragma unroll
        for (int pg = 0; pg < 8; ++pg) {
          const int page = min(kv_beg / 16 + j * 8 + pg, last_page);   // pages past the end are masked
          int b = page < p.bt_stride ? bt[page] : -1;
          if (b < 0 || b >= p.num_blocks) {
            set_status(p.status, kBadArgument);
            b = 0;
          }
          blk[pg] = b;
        }
        mbar_arrive_expect_tx(&k_full[s], 2 * kTile);
#pragma unroll
        for (int pg = 0; pg < 8; ++pg)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_4d(sK + (s * 2 + h) * kTile + pg * 2048, &tmK, &k_full[s], h * 64, 0, kvh, blk[pg]);
        mbar_arrive_expect_tx(&v_full[s], 2 * kTile);
#pragma unroll
        for (int pg = 0; pg < 8; ++pg)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_4d(sV + (s * 2 + h) * kTile + pg * 2048, &tmV, &v_full[s], h * 64, 0, kvh, blk[pg]);
      }
      // drain: every filled stage has been consumed before the CTA exits
      for (int j = max(0, ntiles - 2); j < ntiles; ++j)
        if (!mbar_wait(&kv_empty[j & 1], (j >> 1) & 1, p.status, kAttnTimeout)) break;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(128, 128);
      constexpr uint32_t idesc_pv = idesc_bf16(128, 128) | (1u << 16);   // B (V) MN-major
      const uint32_t tO = tmem_base + 256;
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1, u = j >> 1;
        if (j >= 2 && !mbar_wait(&s_empty[s], (u - 1) & 1, p.status, kAttnTimeout)) return false;
        if (!mbar_wait(&k_full[s], u & 1, p.status, kAttnTimeout)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t dq = smem_desc_k_sw128(smem_u32(sQ + (kk >> 2) * kTile)) + 2 * (kk & 3);
          const uint64_t dk = smem_desc_k_sw128(smem_u32(sK + (s * 2 + (kk >> 2)) * kTile)) + 2 * (kk & 3);
          umma_f16(tmem_base + s * 128, dq, dk, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        return true;
      };
      bool ok = issue_s(0);
      for (int j = 0; j < ntiles && ok; ++j) {
        if (j + 1 < ntiles && !(ok = issue_s(j + 1))) break;
        const int s = j & 1;
        if (!mbar_wait(&p_full[s], (j >> 1) & 1, p.status, kAttnTimeout)) { ok = false; break; }
        if (!mbar_wait(&v_full[s], (j >> 1) & 1, p.status, kAttnTimeout)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // P of kv positions [16 kk, 16 kk + 16): bf16 pairs in TMEM, the first 64 kv in
          // columns [0, 32) of the slot, the second 64 in [64, 96) (each softmax thread's half)
          const uint32_t tp = tmem_base + s * 128 + (kk >> 2) * 64 + (kk & 3) * 8;
          const uint64_t dv = smem_desc_mn_sw128(smem_u32(sV + (s * 2) * kTile + kk * 2048), kTile);
          umma_f16_ts(tO, tp, dv, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[s]);
        umma_commit(&s_empty[s]);
        umma_commit(pv_done);
      }
      umma_commit(o_full);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    // warps 2..9: lane quarter = warp & 3 gives the row, (warp - 2) / 4 the 64-column half
    const int quarter = warp & 3;
    const int hc = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int t = r / a.G, g = r % a.G;
    const int pos = ctx + tok0 + t;
    const int lo = WINDOW ? pos - p.window + 1 : -0x40000000;   // valid kv positions: [lo, pos]
    const float l2e = 1.4426950408889634f;
    const float sc = p.scale * l2e;
    const float ab = ALIBI ? p.alibi[kvh * a.G + g] * l2e : 0.f;   // ALiBi slope, log2 domain
    float m_use = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], (j >> 1) & 1, p.status, kAttnTimeout)) { ok = false; break; }
      tc_fence_after();
      float x[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tmem_base + lane_off + s * 128 + hc * 64 + c * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(u[i]);
      }
      const int c0 = kv_beg + j * 128 + hc * 64;     // kv position of x[0]
      float mx = -INFINITY;
      if (!SOFTCAP && !ALIBI && c0 >= lo && c0 + 63 <= pos) {  // interior tile: nothing masked
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          x[c] *= sc;
          mx = fmaxf(mx, x[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          float v = x[c];
          if (SOFTCAP) v = p.softcap * tanhf(v * p.scale / p.softcap) * l2e;
          else v *= sc;
          const int kp = c0 + c;
          if (ALIBI) v += ab * static_cast<float>(kp - pos);
          v = (kp >= lo && kp <= pos) ? v : -INFINITY;
          x[c] = v;
          mx = fmaxf(mx, v);
        }
      }
      // row maximum = max of the two half rows (exchanged through shared memory)
      xch[(s * 2 + hc) * 128 + r] = mx;
      mbar_arrive(mx_bar);
      if (!mbar_wait(mx_bar, j & 1, p.status, kAttnTimeout)) { ok = false; break; }
      mx = fmaxf(mx, xch[(s * 2 + (hc ^ 1)) * 128 + r]);
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_use + 8.f) {               // also the first finite maximum (m_use = -inf)
        alpha = m_use == -INFINITY ? 0.f : exp2f(m_use - mx);
        rescale = j > 0 && m_use != -INFINITY;
        m_use = mx;
      }
      float rs = 0.f;
      uint32_t pk[32];
      if (m_use == -INFINITY) {
#pragma unroll
        for (int c = 0; c < 32; ++c) pk[c] = 0u;
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(exp2f(x[2 * c] - m_use), exp2f(x[2 * c + 1] - m_use));
          const float2 f = __bfloat1622float2(b2);
          rs += f.x + f.y;                   // sum what the MMA will see
          pk[c] = *reinterpret_cast<const uint32_t*>(&b2);
        }
      }
      l = l * alpha + rs;
      // tcgen05.ld/st are warp-collective: the warp rescales if any of its rows needs it,
      // after the previous PV (which accumulates into O) completed
      if (__any_sync(0xffffffffu, rescale)) {
        if (j > 0 && !mbar_wait(pv_done, (j - 1) & 1, p.status, kAttnTimeout)) { ok = false; break; }
        tc_fence_after();
        if (!rescale) alpha = 1.f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t u[32];
          const uint32_t ta = tmem_base + lane_off + 256 + hc * 64 + c * 32;
          tmem_ld_32x32b_x32(ta, u);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
          tmem_st_32x32b_x32(ta, u);
        }
        tmem_st_wait();
      }
      // P into this thread's own S columns (already read into x): the PV MMA's A operand
      tmem_st_32x32b_x32(tmem_base + lane_off + s * 128 + hc * 64, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[s]);
    }
    // row sum = sum of the two half rows
    xsum[hc * 128 + r] = l;
    mbar_arrive(fin_bar);
    if (ok && mbar_wait(fin_bar, 0, p.status, kAttnTimeout) && mbar_wait(o_full, 0, p.status, kAttnTimeout)) {
      l += xsum[(hc ^ 1) * 128 + r];
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = p.out + static_cast<size_t>(q0 + tok0 + min(t, ntok - 1)) * p.out_stride +
                           (kvh * a.G + g) * D + hc * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tmem_base + lane_off + 256 + hc * 64 + c * 32, u);   // warp-collective
        tmem_ld_wait();
        if (t < ntok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 o;
            __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              oh[k] = __floats2bfloat162_rn(__uint_as_float(u[i + 2 * k]) * inv,
                                            __uint_as_float(u[i + 2 * k + 1]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + i) = o;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

// ---------------------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// paged cache [blocks][Hkv][16][128] (block stride in elements) as a 4-D map, box = 64 d x 16 slots
static int make_tmap_paged(CUtensorMap* m, const void* cache, int num_blocks, int hkv, int64_t block_stride) {
  auto fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[4] = {128, 16, static_cast<cuuint64_t>(hkv), static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[3] = {128 * 2, 16 * 128 * 2, static_cast<cuuint64_t>(block_stride) * 2};
  cuuint32_t box[4] = {64, 16, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(cache), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

bool prefill_tc_supported(const PrefillAttnParams& p) {
  if (p.head_dim != 128 || p.num_kv_heads <= 0 || p.num_q_heads % p.num_kv_heads) return false;
  if (p.alibi != nullptr && p.softcap > 0.f) return false;
  const int G = p.num_q_heads / p.num_kv_heads;
  return G >= 1 && G <= 128 && 128 % G == 0 && (p.block_stride * 2) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(p.k_cache) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.v_cache) & 15) == 0;
}

int prefill_tc_launch(const PrefillAttnParams& p, cudaStream_t st) {
  if (p.num_seqs == 0) return 0;
  PfTcArgs a{};
  a.p = p;
  a.G = p.num_q_heads / p.num_kv_heads;
  a.tq = 128 / a.G;
  a.tiles_per_seq = (p.max_q_len + a.tq - 1) / a.tq;
  CUtensorMap tk, tv;
  if (make_tmap_paged(&tk, p.k_cache, p.num_blocks, p.num_kv_heads, p.block_stride)) return -2;
  if (make_tmap_paged(&tv, p.v_cache, p.num_blocks, p.num_kv_heads, p.block_stride)) return -3;
  dim3 grid(p.num_seqs * a.tiles_per_seq, p.num_kv_heads);
#define RZ_PF(SC, WIN, AL)                                                                                \
  {                                                                                                       \
    opt_in_smem<prefill_tc_kernel<SC, WIN, AL>>(kPfSmem);                                                 \
    prefill_tc_kernel<SC, WIN, AL><<<grid, kPfThreads, kPfSmem, st>>>(tk, tv, a);                         \
  }
  const bool sc = p.softcap > 0.f, win = p.window > 0, al = p.alibi != nullptr;
  if (al && win) RZ_PF(false, true, true)
  else if (al) RZ_PF(false, false, true)
  else if (sc && win) RZ_PF(true, true, false)
  else if (sc) RZ_PF(true, false, false)
  else if (win) RZ_PF(false, true, false)
  else RZ_PF(false, false, false)
#undef RZ_PF
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz
