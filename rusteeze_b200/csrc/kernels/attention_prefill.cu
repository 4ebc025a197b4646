// Varlen prefill / chunked-prefill / verify attention over the paged KV cache.
//
// Queries of a sequence are the LAST q_len positions of its context; keys are
// read from the paged cache (the new tokens' K/V were written by
// rope_and_cache first), so prefix-cached pages, chunked prefill and
// speculative verification (q_len = k+1) all use this one kernel.  Masks
// (causal, sliding window, soft-cap) are applied in registers -- nothing is
// materialised on the host, unlike the reference (crates/rusteeze-model/src/
// architectures/common.rs:365-413, mistral.rs:334-363).
//
// Grid (q tiles of 64, Hq, prefill sequences); 4 warps x 16 query rows.
// K/V tiles of 64 tokens (4 pages) stream through a double-buffered,
// XOR-swizzled shared-memory ring with cp.async; S = QK^T and O += PV run on
// mma.sync m16n8k16 (bf16 in, fp32 accumulate) with an online softmax in
// registers (FlashAttention-2 dataflow; the reference's CPU version is
// crates/rusteeze-engine/src/flash_attention.rs:186-318).
#include "attention.h"
#include "common.cuh"

namespace rz {

constexpr int kPBQ = 64;
constexpr int kPBKV = 64;

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// byte offset of (row, 16-byte chunk) inside a [rows][D] bf16 tile with XOR swizzle
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(128) prefill_attn_kernel(PrefillAttnParams p) {
  constexpr int kTile = kPBKV * D * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kPBQ * D * 2;     // 2 buffers
  uint8_t* sV = sK + 2 * kTile;          // 2 buffers
  const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV);

  const int seq = p.seq_offset + blockIdx.z;
  const int qh = blockIdx.y;
  const int kvh = qh / (p.num_q_heads / p.num_kv_heads);
  const int qt = blockIdx.x;
  const int q0 = p.query_start_loc[seq];
  const int q_len = p.query_start_loc[seq + 1] - q0;
  if (qt * kPBQ >= q_len) return;
  const int L = p.seq_lens[seq];
  if (L > p.bt_stride * 16 || q_len > L) {  // inconsistent metadata: record and skip this tile
    set_status(p.status, kBadArgument);
    return;
  }
  const int ctx0 = L - q_len;
  const int rows_valid = min(kPBQ, q_len - qt * kPBQ);
  const int qpos_lo = ctx0 + qt * kPBQ;
  const int qpos_hi = qpos_lo + rows_valid - 1;
  const int kv_end = qpos_hi + 1;
  int kv_begin = 0;
  if (p.window > 0) kv_begin = max(0, qpos_lo - p.window + 1);
  const int t_begin = kv_begin / kPBKV;
  const int t_end = (kv_end + kPBKV - 1) / kPBKV;
  const int nblk = (L + 15) / 16;
  const int32_t* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kChunks = D / 8;

  // ---- Q tile -> smem
  for (int i = tid; i < kPBQ * kChunks; i += 128) {
    const int r = i / kChunks, c = i % kChunks;
    uint32_t dst = aQ + swz<D>(r, c);
    if (r < rows_valid) {
      const __nv_bfloat16* src = p.q + static_cast<int64_t>(q0 + qt * kPBQ + r) * p.q_stride + qh * D + c * 8;
      cp_async16(dst, src);
    } else {
      *reinterpret_cast<uint4*>(sQ + swz<D>(r, c)) = make_uint4(0, 0, 0, 0);
    }
  }
  auto load_kv = [&](int tile, int buf) {
    for (int i = tid; i < kPBKV * kChunks; i += 128) {
      const int r = i / kChunks, c = i % kChunks;
      int page = tile * 4 + r / 16;
      page = page < nblk ? page : nblk - 1;   // beyond the context: any valid page (masked later)
      int64_t pid = bt[page];
      if (pid < 0 || pid >= p.num_blocks) {   // corrupt block table: record and read page 0 instead
        set_status(p.status, kBadArgument);
        pid = 0;
      }
      const int64_t off = pid * p.block_stride +
                          (static_cast<int64_t>(kvh) * 16 + (r & 15)) * D + c * 8;
      cp_async16(aK + buf * kTile + swz<D>(r, c), p.k_cache + off);
      cp_async16(aV + buf * kTile + swz<D>(r, c), p.v_cache + off);
    }
  };
  load_kv(t_begin, 0);
  cp_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const float sl2 = p.scale * 1.4426950408889634f;  // scale * log2(e)
  const float ab = p.alibi != nullptr ? p.alibi[qh] * 1.4426950408889634f : 0.f;  // ALiBi slope, log2
  const int row_a = warp * 16 + (lane >> 2);          // this thread's rows: row_a, row_a + 8
  const int qpos_a = qpos_lo + row_a;

  for (int t = t_begin; t < t_end; ++t) {
    const int buf = (t - t_begin) & 1;
    if (t + 1 < t_end) {
      load_kv(t + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    // ---- S = Q K^T  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(aQ + swz<D>(warp * 16 + (lane & 15), 2 * kk + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int krow = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int kch = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(aK + buf * kTile + swz<D>(krow, kch), b0, b1, b2, b3);
        mma16816(s[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- mask + online softmax (log2 domain)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kpos = t * kPBKV + nt * 8 + 2 * (lane & 3) + (e & 1);
        const int qpos = qpos_a + ((e >> 1) << 3);
        float v = s[nt][e];
        if (p.softcap > 0.f) v = p.softcap * tanhf(v * p.scale / p.softcap) * 1.4426950408889634f;
        else v *= sl2;
        v += ab * static_cast<float>(kpos - qpos);
        bool masked = kpos > qpos || (p.window > 0 && kpos <= qpos - p.window);
        v = masked ? -INFINITY : v;
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
    for (int nt = 0; nt < 8; ++nt) {
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
    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dn = 0; dn < D / 16; ++dn) {
        uint32_t b0, b1, b2, b3;
        const int vrow = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int vch = 2 * dn + (lane >> 4);
        ldsm_x4_t(aV + buf * kTile + swz<D>(vrow, vch), b0, b1, b2, b3);
        mma16816(o[2 * dn], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * dn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  // ---- finalise
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = row_a + h * 8;
    if (r >= rows_valid) continue;
    const float inv = l_r[h] > 0.f ? 1.f / l_r[h] : 0.f;
    __nv_bfloat16* dst = p.out + static_cast<int64_t>(q0 + qt * kPBQ + r) * p.out_stride + qh * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const int d = i * 8 + 2 * (lane & 3);
      *reinterpret_cast<__nv_bfloat162*>(dst + d) = __floats2bfloat162_rn(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
    }
  }
}

template <int D>
static int launch_prefill(const PrefillAttnParams& p, cudaStream_t st) {
  constexpr int smem = kPBQ * D * 2 + 4 * kPBKV * D * 2;
  opt_in_smem<prefill_attn_kernel<D>>(smem);
  dim3 grid((p.max_q_len + kPBQ - 1) / kPBQ, p.num_q_heads, p.num_seqs);
  prefill_attn_kernel<D><<<grid, 128, smem, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------- fp8 cache -> bf16
// Grid (num_seqs, kGatherSplit): CTA (i, y) takes pages y, y + kGatherSplit, ... of sequence
// seq_offset + i.  Its scratch row offset is the sum of ceil(len / 16) over the earlier
// sequences, summed by the CTA itself (a few hundred lengths at most).
constexpr int kGatherSplit = 16;
constexpr int kGatherThreads = 256;

template <int KVF>
__device__ __forceinline__ void fp8x8_to_bf16(uint2 raw, float scale, __nv_bfloat16* dst) {
  const __nv_fp8_interpretation_t fmt = KVF == kKvE4m3 ? __NV_E4M3 : __NV_E5M2;
  const uint32_t w[2] = {raw.x, raw.y};
  __align__(16) __nv_bfloat162 out[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>((w[k >> 1] >> (16 * (k & 1))) & 0xffffu), fmt);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
    out[k] = __floats2bfloat162_rn(f.x * scale, f.y * scale);
  }
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(out);
}

template <int KVF>
__global__ void __launch_bounds__(kGatherThreads) kv_dequant_gather_kernel(
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out, int32_t* __restrict__ bt_out,
    int64_t bt_out_stride, const uint8_t* __restrict__ k_cache, const uint8_t* __restrict__ v_cache,
    int64_t block_stride, int num_blocks, const int32_t* __restrict__ block_tables, int64_t bt_stride,
    const int32_t* __restrict__ seq_lens, int seq_offset, int Hkv, int D, float k_scale, float v_scale,
    int64_t out_blocks, int* status) {
  __shared__ int64_t red[kGatherThreads / 32];
  const int i = blockIdx.x;
  const int seq = seq_offset + i;
  int64_t part = 0;
  for (int k = threadIdx.x; k < i; k += blockDim.x) part += (max(seq_lens[seq_offset + k], 0) + 15) / 16;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
  __syncthreads();
  int64_t base = 0;
#pragma unroll
  for (int w = 0; w < kGatherThreads / 32; ++w) base += red[w];
  int L = seq_lens[seq];
  if (L < 0 || L > bt_stride * 16 || L > bt_out_stride * 16) {
    if (threadIdx.x == 0) set_status(status, kBadArgument);
    L = 0;
  }
  const int nblk = (L + 15) / 16;
  const int64_t page_elems = static_cast<int64_t>(Hkv) * 16 * D;   // one block of one layer
  const int chunks = static_cast<int>(page_elems / 8);
  for (int b = blockIdx.y; b < nblk; b += gridDim.y) {
    const int64_t dst_blk = base + b;
    if (dst_blk >= out_blocks) {          // scratch sized by the caller from the same lengths
      if (threadIdx.x == 0) set_status(status, kBadArgument);
      return;
    }
    int64_t pid = block_tables[static_cast<int64_t>(seq) * bt_stride + b];
    if (pid < 0 || pid >= num_blocks) {
      if (threadIdx.x == 0) set_status(status, kBadArgument);
      pid = 0;
    }
    if (threadIdx.x == 0) bt_out[static_cast<int64_t>(seq) * bt_out_stride + b] = static_cast<int32_t>(dst_blk);
    const uint8_t* ks = k_cache + pid * block_stride;
    const uint8_t* vs = v_cache + pid * block_stride;
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      fp8x8_to_bf16<KVF>(*reinterpret_cast<const uint2*>(ks + c * 8), k_scale, k_out + dst_blk * page_elems + c * 8);
      fp8x8_to_bf16<KVF>(*reinterpret_cast<const uint2*>(vs + c * 8), v_scale, v_out + dst_blk * page_elems + c * 8);
    }
  }
}

int kv_dequant_gather_launch(__nv_bfloat16* k_out, __nv_bfloat16* v_out, int32_t* bt_out, int64_t bt_out_stride,
                             const uint8_t* k_cache, const uint8_t* v_cache, int64_t block_stride, int num_blocks,
                             const int32_t* block_tables, int64_t bt_stride, const int32_t* seq_lens,
                             int seq_offset, int num_seqs, int Hkv, int D, int kv_fmt, float k_scale,
                             float v_scale, int64_t out_blocks, int* status, cudaStream_t st) {
  if (num_seqs == 0) return 0;
  if (D % 16 || block_stride % 8 || (reinterpret_cast<uintptr_t>(k_cache) & 7) ||
      (reinterpret_cast<uintptr_t>(v_cache) & 7))
    return -1;
  const dim3 grid(num_seqs, kGatherSplit);
  if (kv_fmt == kKvE4m3)
    kv_dequant_gather_kernel<kKvE4m3><<<grid, kGatherThreads, 0, st>>>(
        k_out, v_out, bt_out, bt_out_stride, k_cache, v_cache, block_stride, num_blocks, block_tables, bt_stride,
        seq_lens, seq_offset, Hkv, D, k_scale, v_scale, out_blocks, status);
  else if (kv_fmt == kKvE5m2)
    kv_dequant_gather_kernel<kKvE5m2><<<grid, kGatherThreads, 0, st>>>(
        k_out, v_out, bt_out, bt_out_stride, k_cache, v_cache, block_stride, num_blocks, block_tables, bt_stride,
        seq_lens, seq_offset, Hkv, D, k_scale, v_scale, out_blocks, status);
  else
    return -1;
  return static_cast<int>(cudaGetLastError());
}

int prefill_attention_launch(const PrefillAttnParams& p, cudaStream_t st) {
  if (p.num_seqs == 0) return 0;
  switch (p.head_dim) {
    case 64: return launch_prefill<64>(p, st);
    case 128: return launch_prefill<128>(p, st);
    case 256: return launch_prefill<256>(p, st);
    default: return -100;
  }
}

}  // namespace rz
