// Block-scaled FP8 GEMM on 5th-generation tensor cores:
//   D[M,N] = sum_kb (Aq_kb * Bq_kb^T) * a_scale[kb][m] * b_scale[n/128][kb]
// Aq: e4m3 activations quantised 1x128 (per row, per 128-wide K block),
// Bq: e4m3 weights quantised 128x128, scales fp32 -- the format of the
// block-scaled checkpoints (the reference's quantizers are CPU-only and
// dequantise before every matmul, crates/rusteeze-tensor/src/quantize.rs:
// 292-308).
//
// tcgen05 block-scaled MMA kinds take power-of-two (UE8M0) scales per 32 K
// elements, which cannot carry arbitrary fp32 scales, so the scales are
// applied by "promotion": each 128-wide K block is accumulated by
// unscaled `tcgen05.mma.kind::f8f6f4` (M=128, N=128, K=32, 4 per block) into
// a fresh TMEM partial; 8 epilogue warps read the partial (tcgen05.ld),
// multiply by a_scale[row] * b_scale and add it into fp32 registers.  The
// partial is double buffered in TMEM so the MMAs of block kb+1 overlap the
// promotion of block kb.
//
// Warps: 0 = TMA producer (no cluster multicast), 1 = TMEM alloc + MMA
// issue, 2..9 = epilogue (warp w reads TMEM lanes 32*(w%4).., columns
// 64*((w-2)/4)..).  Epilogues: bias, residual, SiLU(gate)*up on
// 64-row interleaved gate/up weights, or fp32 split-K partials.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm_bf16.h"
#include "gemm_fp8.h"

namespace rz {

namespace {
constexpr int kF8BM = 128, kF8BN = 128, kF8BK = 128;  // K block = one scale block = one 128-byte row
constexpr int kF8Stages = 6;
constexpr int kF8ABytes = kF8BM * kF8BK;
constexpr int kF8BBytes = kF8BN * kF8BK;
constexpr int kF8StageBytes = kF8ABytes + kF8BBytes;
constexpr int kF8Parts = 4;          // TMEM partial accumulators in flight (4 x 128 columns = all of TMEM)
constexpr int kF8Threads = 320;
constexpr int kF8EpiThreads = 256;
constexpr int kF8Smem = kF8Stages * kF8StageBytes + 1024 + 256;
}  // namespace

__device__ __forceinline__ float f8_silu(float x) { return x / (1.0f + __expf(-x)); }


__global__ void __launch_bounds__(kF8Threads, 1)
    gemm_fp8_tcgen05(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     Fp8GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t* smA = smem;
  uint8_t* smB = smem + kF8Stages * kF8ABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kF8Stages * kF8StageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kF8Stages;
  uint64_t* pfull = bars + 2 * kF8Stages;
  uint64_t* pempty = pfull + kF8Parts;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pempty + kF8Parts);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.m_tiles * p.n_tiles * p.k_splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kF8Stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kF8Parts; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], kF8EpiThreads);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kF8Parts * kF8BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int ks = u % p.k_splits, t = u / p.k_splits;
        const int mb = t % p.m_tiles, nb = t / p.m_tiles;
        const int kb0 = ks * p.kb_per_split, kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, kGemmProducerTimeout)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], kF8StageBytes);
          tma_load_2d(smA + s * kF8ABytes, &tmA, &full[s], kb * kF8BK, mb * kF8BM);
          tma_load_2d(smB + s * kF8BBytes, &tmB, &full[s], kb * kF8BK, nb * kF8BN);
          if (++s == kF8Stages) { s = 0; ph ^= 1; }
        }
      }
      for (int i = 0; i < kF8Stages && ok; ++i) {
        if (!mbar_wait(&empty[s], ph ^ 1, p.status, kGemmProducerTimeout)) break;
        if (++s == kF8Stages) { s = 0; ph ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3(kF8BM, kF8BN);
      int s = 0, buf = 0;
      uint32_t ph = 0, bph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int ks = u % p.k_splits;
        const int kb0 = ks * p.kb_per_split, kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&pempty[buf], bph ^ 1, p.status, kGemmMmaTimeout)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, p.status, kGemmMmaTimeout)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = smem_desc_k_sw128(smem_u32(smA + s * kF8ABytes));
          const uint64_t db = smem_desc_k_sw128(smem_u32(smB + s * kF8BBytes));
          const uint32_t dtm = tmem_base + buf * kF8BN;
#pragma unroll
          for (int k = 0; k < kF8BK / 32; ++k)   // 32 e4m3 = 32 bytes per MMA: +2 in the >>4 address field
            umma_f8(dtm, da + 2 * k, db + 2 * k, idesc, k > 0 ? 1u : 0u);
          umma_commit(&empty[s]);
          umma_commit(&pfull[buf]);
          if (++s == kF8Stages) { s = 0; ph ^= 1; }
          if (++buf == kF8Parts) { buf = 0; bph ^= 1; }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue / promotion
    // Warp w owns TMEM lanes 32*(w%4).. (its rows) and, with h = (w-2)/4, the column groups
    // [32h, 32h+32) and [64+32h, 64+32h+32) of the 128-wide tile.  With gate/up rows
    // interleaved in 64-row blocks those are matching gate and up columns, so the SiLU
    // epilogue needs no exchange between warps.
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int h = ew >> 2;
    const int row_in_tile = quarter * 32 + lane;
    int buf = 0;
    uint32_t bph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int ks = u % p.k_splits, t = u / p.k_splits;
      const int mb = t % p.m_tiles, nb = t / p.m_tiles;
      const int kb0 = ks * p.kb_per_split, kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
      const int row = mb * kF8BM + row_in_tile;
      const bool row_ok = row < p.M;
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
      const float* a_col = p.a_scale + (row_ok ? row : 0);
      const float* b_row = p.b_scale + static_cast<int64_t>(nb) * p.b_scale_ld;
      // scales of the next k-block are loaded before waiting on the current partial
      float sa_n = kb0 < kb1 ? a_col[static_cast<int64_t>(kb0) * p.a_scale_ld] : 0.f;
      float sb_n = kb0 < kb1 ? b_row[kb0] : 0.f;
      for (int kb = kb0; kb < kb1; ++kb) {
        const float sc = (row_ok ? sa_n : 0.f) * sb_n;
        if (kb + 1 < kb1) {
          sa_n = a_col[static_cast<int64_t>(kb + 1) * p.a_scale_ld];
          sb_n = b_row[kb + 1];
        }
        if (!mbar_wait(&pfull[buf], bph, p.status, kGemmEpilogueTimeout)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * kF8BN;
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(taddr + 32 * h, r0);
        tmem_ld_32x32b_x32(taddr + 64 + 32 * h, r1);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&pempty[buf]);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          acc[j] = fmaf(__uint_as_float(r0[j]), sc, acc[j]);
          acc[32 + j] = fmaf(__uint_as_float(r1[j]), sc, acc[32 + j]);
        }
        if (++buf == kF8Parts) { buf = 0; bph ^= 1; }
      }
      if (!ok || !row_ok) continue;
      const int cA = nb * kF8BN + 32 * h;        // first column group
      const int cB = cA + 64;                    // second column group
      if (cA >= p.N) continue;
      if (p.k_splits > 1) {
        float* dst = p.partial + (static_cast<size_t>(ks) * p.M + row) * p.N;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          *reinterpret_cast<float4*>(dst + cA + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
          *reinterpret_cast<float4*>(dst + cB + j) =
              make_float4(acc[32 + j], acc[33 + j], acc[34 + j], acc[35 + j]);
        }
      } else if (p.epi == kEpiSiluMul) {
        __nv_bfloat16* dst = p.D + static_cast<size_t>(row) * p.ldd + nb * (kF8BN / 2) + 32 * h;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float g0 = acc[j], g1 = acc[j + 1], u0 = acc[32 + j], u1 = acc[33 + j];
          if (p.bias) {
            g0 += bf2f(p.bias[cA + j]);
            g1 += bf2f(p.bias[cA + j + 1]);
            u0 += bf2f(p.bias[cB + j]);
            u1 += bf2f(p.bias[cB + j + 1]);
          }
          *reinterpret_cast<__nv_bfloat162*>(dst + j) = __floats2bfloat162_rn(f8_silu(g0) * u0, f8_silu(g1) * u1);
        }
      } else {
        __nv_bfloat16* dst = p.D + static_cast<size_t>(row) * p.ldd;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int c0 = g ? cB : cA;
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float a = acc[32 * g + j], b = acc[32 * g + j + 1];
            if (p.bias) {
              a += bf2f(p.bias[c0 + j]);
              b += bf2f(p.bias[c0 + j + 1]);
            }
            if (p.residual) {
              const __nv_bfloat16* rr = p.residual + static_cast<size_t>(row) * p.ldr + c0 + j;
              a += bf2f(rr[0]);
              b += bf2f(rr[1]);
            }
            *reinterpret_cast<__nv_bfloat162*>(dst + c0 + j) = __floats2bfloat162_rn(a, b);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kF8Parts * kF8BN);
}

// ---------------------------------------------------------------------------- activation quant
// One warp per (row, 128-wide K group): amax -> scale = amax / 448 -> e4m3.
__global__ void quant_fp8_act_kernel(__nv_fp8_e4m3* __restrict__ xq, float* __restrict__ xs,
                                     const __nv_bfloat16* __restrict__ x, int M, int K, int64_t ldx, int64_t xs_ld) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int groups = K / 128;
  if (wid >= static_cast<int64_t>(M) * groups) return;
  const int row = static_cast<int>(wid / groups), g = static_cast<int>(wid % groups);
  const __nv_bfloat16* src = x + row * ldx + g * 128 + lane * 4;
  float v[4];
  const __nv_bfloat162 a = reinterpret_cast<const __nv_bfloat162*>(src)[0];
  const __nv_bfloat162 b = reinterpret_cast<const __nv_bfloat162*>(src)[1];
  v[0] = __low2float(a);
  v[1] = __high2float(a);
  v[2] = __low2float(b);
  v[3] = __high2float(b);
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max(amax);
  amax = fmaxf(amax, 1e-12f);
  const float scale = amax / 448.f;
  const float inv = 448.f / amax;
  __nv_fp8_e4m3 q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = __nv_fp8_e4m3(fminf(fmaxf(v[i] * inv, -448.f), 448.f));
  *reinterpret_cast<uint32_t*>(xq + static_cast<int64_t>(row) * K + g * 128 + lane * 4) =
      *reinterpret_cast<uint32_t*>(q);
  if (lane == 0) xs[static_cast<int64_t>(g) * xs_ld + row] = scale;
}

int quant_fp8_act_launch(void* xq, float* xs, const __nv_bfloat16* x, int M, int K, int64_t ldx, int64_t xs_ld,
                         cudaStream_t st) {
  if (M == 0) return 0;
  if (K % 128) return -1;
  const int64_t warps = static_cast<int64_t>(M) * (K / 128);
  const int tb = 256;
  quant_fp8_act_kernel<<<static_cast<int>((warps * 32 + tb - 1) / tb), tb, 0, st>>>(
      reinterpret_cast<__nv_fp8_e4m3*>(xq), xs, x, M, K, ldx, xs_ld);
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------- host
int gemm_fp8_launch(const Fp8GemmParams& p_in, const void* A, int lda, const void* B, int ldb, cudaStream_t st) {
  Fp8GemmParams p = p_in;
  if (p.K % kF8BK) return -1;
  p.k_blocks = p.K / kF8BK;
  p.m_tiles = (p.M + kF8BM - 1) / kF8BM;
  p.n_tiles = (p.N + kF8BN - 1) / kF8BN;
  if (p.k_splits < 1) p.k_splits = 1;
  p.kb_per_split = (p.k_blocks + p.k_splits - 1) / p.k_splits;
  p.k_splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  CUtensorMap ta, tb;
  if (make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.M, p.K, lda, kF8BM, kF8BK)) return -2;
  if (make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.N, p.K, ldb, kF8BN, kF8BK)) return -3;
  opt_in_smem<gemm_fp8_tcgen05>(kF8Smem);
  const int units = p.m_tiles * p.n_tiles * p.k_splits;
  const int grid = units < num_sms() ? units : num_sms();
  gemm_fp8_tcgen05<<<grid, kF8Threads, kF8Smem, st>>>(ta, tb, p);
  if (p.k_splits > 1) {
    GemmParams g{};
    g.M = p.M;
    g.N = p.N;
    g.k_splits = p.k_splits;
    g.D = p.D;
    g.ldd = p.ldd;
    g.partial = p.partial;
    g.bias = p.bias;
    g.residual = p.residual;
    g.ldr = p.ldr;
    g.epi = p.epi;
    const int ncols_out = p.epi == kEpiSiluMul ? p.N / 2 : p.N;
    const long threads = static_cast<long>(p.M) * (ncols_out / 8);
    gemm_splitk_reduce<<<static_cast<int>((threads + 255) / 256), 256, 0, st>>>(g);
  }
  return static_cast<int>(cudaGetLastError());
}

int fp8_plan_splits(int M, int N, int K) {
  const int sms = num_sms();
  const int kblocks = K / kF8BK;
  const int tiles = ((M + kF8BM - 1) / kF8BM) * ((N + kF8BN - 1) / kF8BN);
  int ks = 1;   // enough units to put every SM to work on small-M (weight-streaming) GEMMs
  while (ks < 16 && tiles * ks < sms && kblocks / (ks * 2) >= 2) ks *= 2;
  return ks;
}

}  // namespace rz
