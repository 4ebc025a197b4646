// Tensor-core GEMM on 5th-generation tensor cores: D[M,N] = A[M,K] * B[N,K]^T
// (A = activations, B = nn.Linear-layout weights, both K-major), in two
// operand formats sharing one kernel template:
//   bf16      kind::f16, 64 K-elements (128 bytes) per pipeline stage;
//   MXFP8     kind::mxf8f6f4.block_scale: e4m3 operands, 128 K-elements per
//             stage, one UE8M0 (power-of-two) scale per 32 K-elements of every
//             A row and B row.  The scales travel with each stage (512-byte
//             chunks per 128 rows, already in the tensor-memory copy layout),
//             are moved to TMEM by tcgen05.cp and applied inside the MMA, so
//             the accumulator needs no per-block promotion.
//
// Structure (one persistent CTA per SM, 320 threads, warp-specialised):
//   warp 0      TMA producer: 128-row A tile + BN-row B tile per stage into a
//               STAGES-deep shared-memory ring (128-byte swizzle), plus the
//               scale chunks (bulk copies) for MXFP8; no cluster multicast
//               (each CTA loads its own tiles; reuse comes from L2).
//   warp 1      allocates TMEM (double-buffered BN-column fp32 accumulator;
//               MXFP8 with BN=256 keeps one accumulator so the scale columns
//               fit) and issues the MMAs (M=128, N=BN) from one thread;
//               tcgen05.commit releases smem stages and signals a finished
//               accumulator.
//   warps 2..9  epilogue, two warps per TMEM lane quarter (one accumulator row
//               per thread, half of the tile's columns per warp): the warp
//               copies its share of the accumulator to registers with
//               tcgen05.ld and releases the TMEM buffer at once, then adds
//               bias / residual, applies SiLU(gate)*up on interleaved gate/up
//               weight rows (optionally re-quantising to MXFP8), converts and
//               stores -- overlapping the next tile's MMAs even when there is
//               a single accumulator.
// Work units are (m tile, n tile, k split); m varies fastest so CTAs of one
// wave share the same weight tile through L2.  With k_splits > 1 the
// epilogue writes fp32 partials to a workspace and `gemm_splitk_reduce`
// finishes them (small-M decode GEMMs need the extra parallelism to stream
// weights from all 148 SMs).
//
// Every mbarrier wait is bounded (common.cuh); a timeout records a status
// code and the CTA drains and exits.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm_bf16.h"
#include "mxfp8.cuh"

namespace rz {

constexpr int kBM = 128;
constexpr int kBK = 64;         // bf16 K-elements per stage: one 128-byte swizzle atom
constexpr int kBKMx = 128;      // e4m3 K-elements per stage: the same 128 bytes
constexpr int kSfChunk = 512;   // UE8M0 scales of 128 rows x 4 K-chunks of 32
constexpr int kSfTmemCol = 256; // TMEM column where the MXFP8 scales live
constexpr int kGemmThreads = 320;  // warp 0 TMA producer, warp 1 MMA issuer, warps 2..9 epilogue

template <int BN, bool MX, bool PEER = false>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kABytes = kBM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kSfaBytes = MX ? kSfChunk : 0;
  static constexpr int kSfbBytes = MX ? kSfChunk * (BN / 128) : 0;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;  // bytes landing per stage
  static constexpr int kAccStages = (MX && BN == 256) ? 1 : 2;
  static constexpr int kTmemCols = MX ? 512 : (2 * BN < 32 ? 32 : 2 * BN);
  // epilogue transpose of the peer reduce-scatter instances: 8 warps x 32 rows x 32 bf16
  static constexpr int kOutStageBytes = PEER ? 8 * 32 * 64 : 0;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/ + kOutStageBytes;
  static_assert(!MX || BN >= 128, "MXFP8 tiles cover whole 128-row scale chunks");
  static_assert(kSmemBytes <= 227 * 1024 - 2048, "dynamic + static shared memory must fit one CTA");
  static_assert(!MX || kAccStages * BN <= kSfTmemCol, "accumulators overlap the scale columns");
};

__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* dst, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(dst) = u;
}

__device__ __forceinline__ void load_bf16x8(const __nv_bfloat16* src, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }
// GELU with the tanh approximation (Gemma's GeGLU): 0.5 x (1 + tanh(sqrt(2/pi)(x + 0.044715 x^3)))
__device__ __forceinline__ float gelu_tanh_f(float x) {
  return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}
__device__ __forceinline__ float gate_act(float x, int act) { return act ? gelu_tanh_f(x) : silu(x); }

// What a work unit computes: tile index t (in unit order), K blocks [kb0, kb1) and the split
// index ks of a split-K unit.
struct UnitWork {
  int t, kb0, kb1, ks;
};

__device__ __forceinline__ UnitWork unit_work(const GemmParams& p, int u) {
  UnitWork w;
  w.ks = u % p.k_splits;
  w.t = u / p.k_splits;
  w.kb0 = w.ks * p.kb_per_split;
  w.kb1 = min(p.k_blocks, w.kb0 + p.kb_per_split);
  return w;
}

template <int BN, bool MX, bool PEER>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 GemmParams p) {
  using C = GemmCfg<BN, MX, PEER>;
  constexpr int S = C::kStages;
  constexpr int KS = C::kAccStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * C::kABytes;
  uint8_t* smSfa = smB + S * C::kBBytes;      // 1024-aligned: A/B stage sizes are multiples of 1 KB
  uint8_t* smSfb = smSfa + S * C::kSfaBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  uint64_t* xbar = bars + 2 * S + 5;       // the two epilogue warps of a lane quarter exchange row maxima
  uint4* sm_out = reinterpret_cast<uint4*>(smem + S * C::kStageBytes + 256);
  __shared__ float s_amax[256];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grouped mode (MoE experts): A rows are expert-sorted with every expert's
  // segment starting on a 128-row boundary (grp_off[g], g = 0..G), its valid
  // rows ending at grp_end[g]; B holds G weight matrices of N rows each.  The
  // segment sizes live on the device, so the tile count is read here.
  __shared__ int s_grp[2 * kMaxGemmGroups + 1];
  const int G = p.grp_off ? p.num_groups : 0;
  if (G > 0) {
    for (int i = threadIdx.x; i < 2 * G + 1; i += blockDim.x)
      s_grp[i] = i <= G ? p.grp_off[i] : p.grp_end[i - G - 1];
  }
  const int m_tiles = G ? p.grp_off[G] / kBM : p.m_tiles;
  const int num_units = m_tiles * p.n_tiles * p.k_splits;
  const uint32_t epoch =
      p.epoch_ptr ? *reinterpret_cast<const volatile uint32_t*>(p.epoch_ptr) * 256u + p.call_idx + 1u : 0u;
  // GEMMs that feed or consume a collective finish whole m tiles first: the reduce-scatter
  // consumer and the all-gather producer both work in row blocks
  const bool row_major = p.epi == kEpiPeerRS || p.ag_flag != nullptr;
  pdl_trigger();
  auto group_of = [&](int mb) {
    int g = 0;
    while (g + 1 < G && s_grp[g + 1] <= mb * kBM) ++g;
    return g;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 256);
    }
    mbar_init(xbar, 256);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint64_t ag_ready = 0;                 // m tiles whose all-gathered rows were already seen
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const UnitWork w = unit_work(p, u);
        const int t = w.t;
        const int mb = row_major ? t / p.n_tiles : t % m_tiles;
        const int nb = row_major ? t % p.n_tiles : t / m_tiles;
        const int b_row0 = (G ? group_of(mb) * p.N : 0) + nb * BN;
        if (p.ag_flag && !(mb < 64 && ((ag_ready >> mb) & 1ull))) {
          // all-gathered A rows arrive from their owners: wait (once per m tile) for this
          // tile's row blocks, polling all of its flags together
          const int rb0 = mb * kBM / kAgRowBlock;
          const int rb1 = min((p.ag_rows + kAgRowBlock - 1) / kAgRowBlock, (mb + 1) * kBM / kAgRowBlock);
          ok = wait_flags_geq(p.ag_flag + rb0, rb1 - rb0, epoch, p.status, kCommPeerTimeout);
          fence_proxy_async_global();
          if (!ok) break;
          if (mb < 64) ag_ready |= 1ull << mb;
        }
        const int kb0 = w.kb0, kb1 = w.kb1;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, kGemmProducerTimeout)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          constexpr int kElems = MX ? kBKMx : kBK;
          tma_load_2d(smA + s * C::kABytes, &tmA, &full[s], kb * kElems, mb * kBM);
          tma_load_2d(smB + s * C::kBBytes, &tmB, &full[s], kb * kElems, b_row0);
          if constexpr (MX) {
            bulk_load(smSfa + s * C::kSfaBytes, p.sfa + (static_cast<size_t>(mb) * p.k_blocks + kb) * kSfChunk,
                      kSfChunk, &full[s]);
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              bulk_load(smSfb + s * C::kSfbBytes + j * kSfChunk,
                        p.sfb + (static_cast<size_t>(b_row0 / 128 + j) * p.k_blocks + kb) * kSfChunk,
                        kSfChunk, &full[s]);
          }
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
      // drain: wait until the MMA warp consumed every stage we filled, so no
      // TMA write lands in shared memory after the CTA exits
      for (int i = 0; i < S && ok; ++i) {
        if (!mbar_wait(&empty[s], ph ^ 1, p.status, kGemmProducerTimeout)) break;
        if (++s == S) { s = 0; ph ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, BN);
      const uint32_t tsfa = tmem_base + kSfTmemCol;
      const uint32_t tsfb = tmem_base + kSfTmemCol + 4;
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const UnitWork w = unit_work(p, u);
        const int kb0 = w.kb0, kb1 = w.kb1;
        if (!mbar_wait(&tempty[acc], aph ^ 1, p.status, kGemmMmaTimeout)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dtm = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, p.status, kGemmMmaTimeout)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = smem_desc_k_sw128(smem_u32(smA + s * C::kABytes));
          const uint64_t db = smem_desc_k_sw128(smem_u32(smB + s * C::kBBytes));
          if constexpr (MX) {
            // scales of this stage -> TMEM (ordered before the MMAs below in the tensor pipe)
            tmem_cp_32x128b_warpx4(tsfa, smem_desc_rows16(smem_u32(smSfa + s * C::kSfaBytes)));
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              tmem_cp_32x128b_warpx4(tsfb + 4 * j, smem_desc_rows16(smem_u32(smSfb + s * C::kSfbBytes + j * kSfChunk)));
#pragma unroll
            for (int k = 0; k < kBKMx / 32; ++k) {
              // K-chunk k of 32 e4m3 = +32 bytes (+2 in the >>4 address field); its scales are byte k
              const uint32_t sel = static_cast<uint32_t>(k) << 30;
              umma_mxf8(dtm, da + 2 * k, db + 2 * k, idesc_mxf8(kBM, BN, k), tsfa | sel, tsfb | sel,
                        (kb > kb0 || k > 0) ? 1u : 0u);
            }
          } else {
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              // +32 bytes along K inside the 128-byte swizzle atom = +2 in the >>4 address field
              umma_f16(dtm, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == KS) { acc = 0; aph ^= 1; }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9)
    // Two warps per TMEM lane quarter, each owning half of the tile's columns.  A warp
    // first pulls its whole share of the accumulator into registers and releases the
    // TMEM buffer, then does bias / residual / activation / conversion and the stores
    // while the MMA warp already accumulates the next tile into it.
    // Launched as a programmatic dependent (the all-gather consumer), the TMA and MMA
    // warps start on gathered rows while the previous kernels still run, but nothing is
    // stored before they completed: the output and split-K buffers come from the caching
    // allocator, which may hand out memory those kernels still read.
    if (p.ag_flag) pdl_wait();
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;       // column half of the tile
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t aph = 0;
    uint32_t xph = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const UnitWork w = unit_work(p, u);
      const int ks = w.ks;
      const int t = w.t;
      const int mb = row_major ? t / p.n_tiles : t % m_tiles;
      const int nb = row_major ? t % p.n_tiles : t / m_tiles;
      if (!mbar_wait(&tfull[acc], aph, p.status, kGemmEpilogueTimeout)) break;
      tc_fence_after();
      const int row = mb * kBM + row_in_tile;
      const bool row_ok = row < (G ? s_grp[G + 1 + group_of(mb)] : p.M);
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      if (p.k_splits == 1 && (p.epi == kEpiSiluMul || p.epi == kEpiSiluMulMx)) {
        // (split-K partials always take the raw fp32 path below; the reduce kernel applies the epilogue)
        // gate/up rows interleaved in 64-row blocks: tile column pair pr holds [gate 64 | up 64];
        // this warp takes the 32-column sub-chunk `half` of every pair
        constexpr int NI = BN / 128 > 0 ? BN / 128 : 1;
        uint32_t g[NI][32], v[NI][32];
#pragma unroll
        for (int it = 0; it < NI; ++it) {
          tmem_ld_32x32b_x32(tacc + it * 128 + half * 32, g[it]);
          tmem_ld_32x32b_x32(tacc + it * 128 + 64 + half * 32, v[it]);
        }
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        float o[NI][32];
        float amax = 0.f;
#pragma unroll
        for (int it = 0; it < NI; ++it) {
          const int gcol = nb * BN + it * 128 + half * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float a = __uint_as_float(g[it][j]);
            float b = __uint_as_float(v[it][j]);
            if (p.bias && gcol < p.N) {
              a += bf2f(p.bias[gcol + j]);
              b += bf2f(p.bias[gcol + 64 + j]);
            }
            o[it][j] = gate_act(a, p.gate_act) * b;
            amax = fmaxf(amax, fabsf(o[it][j]));
          }
        }
        if (p.epi == kEpiSiluMul) {
#pragma unroll
          for (int it = 0; it < NI; ++it) {
            const int gcol = nb * BN + it * 128 + half * 32;
            const int ocol = nb * (BN / 2) + it * 64 + half * 32;
            if (row_ok && gcol < p.N) {
              __nv_bfloat16* dst = p.D + static_cast<size_t>(row) * p.ldd + ocol;
#pragma unroll
              for (int j = 0; j < 32; j += 8) store_bf16x8(dst + j, o[it] + j);
            }
          }
        } else if constexpr (BN == 256) {
          // SiLU(gate)*up as the next MXFP8 operand: the tile's 128 outputs of this row are one
          // 1x128 scale block, split over the two warps of this lane quarter
          s_amax[half * 128 + row_in_tile] = amax;
          mbar_arrive(xbar);
          if (!mbar_wait(xbar, xph, p.status, kGemmEpilogueTimeout)) break;
          xph ^= 1;
          amax = fmaxf(amax, s_amax[(half ^ 1) * 128 + row_in_tile]);
          float inv;
          const uint32_t e = ue8m0_scale(amax, &inv);
          if (row_ok) {
#pragma unroll
            for (int it = 0; it < NI; ++it) {
              uint8_t* dst = p.q_out + static_cast<size_t>(row) * p.ldd + nb * 128 + it * 64 + half * 32;
#pragma unroll
              for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint2*>(dst + j) = pack_e4m3x8(o[it] + j, inv);
            }
          }
          if (half == 0) {
            // rows past M keep the neutral scale (their operand rows are never loaded as data)
            const int kbo = p.N / 256;      // 128-column scale blocks of the output row
            *reinterpret_cast<uint32_t*>(p.sf_out + (static_cast<size_t>(mb) * kbo + nb) * kSfChunkBytes +
                                         sf_offset(row_in_tile, 0)) = (row_ok ? e : 127u) * 0x01010101u;
          }
        }
      } else {
        constexpr int NC = BN / 64;          // 32-column chunks in this warp's half
        uint32_t r[NC][32];
#pragma unroll
        for (int c = 0; c < NC; ++c) tmem_ld_32x32b_x32(tacc + half * (BN / 2) + c * 32, r[c]);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        const int colh = nb * BN + half * (BN / 2);
        if (p.k_splits > 1) {
          float* dst = p.partial + (static_cast<size_t>(ks) * p.M + row) * p.N;
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const int col0 = colh + c * 32;
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                if (col0 + j < p.N) {
                  float4 f = make_float4(__uint_as_float(r[c][j]), __uint_as_float(r[c][j + 1]),
                                         __uint_as_float(r[c][j + 2]), __uint_as_float(r[c][j + 3]));
                  *reinterpret_cast<float4*>(dst + col0 + j) = f;
                }
              }
            }
          }
        } else if (PEER) {                        // epilogue kEpiPeerRS (the launcher picks PEER by it)
          // reduce-scatter: each row goes to its owner's slot for this rank, over NVLink.
          // Every 32-column chunk is transposed through shared memory (16-byte units
          // XOR-swizzled by row pair, conflict-free both ways) so that 4 lanes store 64
          // contiguous bytes of one row: 64-byte peer writes instead of 16-byte ones.
          uint4* stg = sm_out + (warp - 2) * 128;
          const int r0 = mb * kBM + quarter * 32;
          jitter_ns(p.jitter_ns, epoch, static_cast<uint32_t>(t), static_cast<uint32_t>(warp));
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const int col0 = colh + c * 32;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float o[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(r[c][j * 8 + i]);
              uint4 u;
              __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
              for (int i = 0; i < 4; ++i) h2[i] = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
              stg[lane * 4 + (j ^ ((lane >> 1) & 3))] = u;
            }
            __syncwarp();
#pragma unroll
            for (int ps = 0; ps < 4; ++ps) {
              const int rr = ps * 8 + (lane >> 2), j = lane & 3;
              const int grow = r0 + rr, gcol = col0 + j * 8;
              const uint4 v = stg[rr * 4 + (j ^ ((rr >> 1) & 3))];
              if (grow < p.M && gcol < p.N) {
                const int owner = grow / p.rs_rows;
                *reinterpret_cast<uint4*>(p.rs_slot[owner] +
                                          (static_cast<size_t>(p.tp_rank) * p.rs_rows + (grow - owner * p.rs_rows)) *
                                              p.N + gcol) = v;
              }
            }
            __syncwarp();
          }
          // this warp's 32 rows x half the columns are stored: publish them to each owner they
          // touch (the warp barrier orders all lanes' stores before lane 0's fence + release)
          __syncwarp();
          if (lane == 0 && r0 < p.M) {
            jitter_ns(p.jitter_ns, epoch + 1u, static_cast<uint32_t>(t), static_cast<uint32_t>(warp));
            __threadfence_system();
            const int r1 = min(p.M, r0 + 32) - 1;
            for (int o = r0 / p.rs_rows; o <= r1 / p.rs_rows; ++o)
              st_release_sys_u32(p.rs_flag[o] + ((static_cast<size_t>(mb) * p.n_tiles + nb) * 8 + quarter * 2 + half) *
                                                    p.tp_world + p.tp_rank,
                                 epoch);
          }
        } else if (row_ok) {
          __nv_bfloat16* dst = p.D + static_cast<size_t>(row) * p.ldd;
#pragma unroll
          for (int c = 0; c < NC; ++c) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              const int col = colh + c * 32 + j;
              if (col < p.N) {
                float o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(r[c][j + i]);
                if (p.bias) {
                  float b[8];
                  load_bf16x8(p.bias + col, b);
#pragma unroll
                  for (int i = 0; i < 8; ++i) o[i] += b[i];
                }
                if (p.residual) {
                  float b[8];
                  load_bf16x8(p.residual + static_cast<size_t>(row) * p.ldr + col, b);
#pragma unroll
                  for (int i = 0; i < 8; ++i) o[i] += b[i];
                }
                store_bf16x8(dst + col, o);
              }
            }
          }
        }
      }
      if (++acc == KS) { acc = 0; aph ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
  pdl_wait();   // a programmatic dependent completes only after its primary grid
}

// Sums k-split partials and applies the epilogue.  One thread per 8 output columns.
__global__ void gemm_splitk_reduce(GemmParams p) {
  const int ncols_out = p.epi == kEpiSiluMul ? p.N / 2 : p.N;
  const int vec_per_row = ncols_out / 8;
  const long idx = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<long>(p.M) * vec_per_row) return;
  const int row = static_cast<int>(idx / vec_per_row);
  const int oc = static_cast<int>(idx % vec_per_row) * 8;
  float o[8];
  if (p.epi == kEpiSiluMul) {
    // output col oc -> gate col (oc/64)*128 + oc%64, up col +64
    const int gc = (oc / 64) * 128 + (oc % 64);
    float g[8] = {0}, v[8] = {0};
    for (int k = 0; k < p.k_splits; ++k) {
      const float* src = p.partial + (static_cast<size_t>(k) * p.M + row) * p.N;
      float4 a0 = *reinterpret_cast<const float4*>(src + gc);
      float4 a1 = *reinterpret_cast<const float4*>(src + gc + 4);
      float4 b0 = *reinterpret_cast<const float4*>(src + gc + 64);
      float4 b1 = *reinterpret_cast<const float4*>(src + gc + 68);
      g[0] += a0.x; g[1] += a0.y; g[2] += a0.z; g[3] += a0.w;
      g[4] += a1.x; g[5] += a1.y; g[6] += a1.z; g[7] += a1.w;
      v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
      v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
    }
    for (int i = 0; i < 8; ++i) {
      if (p.bias) {
        g[i] += bf2f(p.bias[gc + i]);
        v[i] += bf2f(p.bias[gc + 64 + i]);
      }
      o[i] = gate_act(g[i], p.gate_act) * v[i];
    }
  } else {
    for (int i = 0; i < 8; ++i) o[i] = 0.f;
    for (int k = 0; k < p.k_splits; ++k) {
      const float* src = p.partial + (static_cast<size_t>(k) * p.M + row) * p.N + oc;
      float4 a0 = *reinterpret_cast<const float4*>(src);
      float4 a1 = *reinterpret_cast<const float4*>(src + 4);
      o[0] += a0.x; o[1] += a0.y; o[2] += a0.z; o[3] += a0.w;
      o[4] += a1.x; o[5] += a1.y; o[6] += a1.z; o[7] += a1.w;
    }
    if (p.bias) {
      float b[8];
      load_bf16x8(p.bias + oc, b);
      for (int i = 0; i < 8; ++i) o[i] += b[i];
    }
    if (p.residual) {
      float b[8];
      load_bf16x8(p.residual + static_cast<size_t>(row) * p.ldr + oc, b);
      for (int i = 0; i < 8; ++i) o[i] += b[i];
    }
  }
  store_bf16x8(p.D + static_cast<size_t>(row) * p.ldd + oc, o);
}

// ---------------------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D K-major tensor map: rows x cols(=K) elements, row stride ld elements,
// box = box_rows x 64 (one 128-byte swizzle atom per row for bf16).
int make_tmap_2d(CUtensorMap* m, const void* ptr, CUtensorMapDataType dt, int elem_bytes, int64_t rows,
                 int64_t cols, int64_t ld, int box_rows, int box_cols) {
  auto fn = get_encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

// SM count of the current device for grid sizing and tile planning; B200's 148 when the
// query fails (no device: plans are still computed, e.g. on a build host)
int num_sms() {
  static std::atomic<int> cached{0};
  int n = cached.load(std::memory_order_relaxed);
  if (n > 0) return n;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 148;
  }
  cached.store(n, std::memory_order_relaxed);
  return n;
}

template <int BN, bool MX, bool PEER>
static int launch_inst(const GemmParams& p0, const void* A, int lda, const void* B, int ldb, cudaStream_t st) {
  using C = GemmCfg<BN, MX, PEER>;
  constexpr int kElems = MX ? kBKMx : kBK;
  const CUtensorMapDataType dt = MX ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int es = MX ? 1 : 2;
  CUtensorMap ta, tb;
  if (make_tmap_2d(&ta, A, dt, es, p0.M, p0.K, lda, kBM, kElems)) return -2;
  if (make_tmap_2d(&tb, B, dt, es, p0.N, p0.K, ldb, BN, kElems)) return -3;
  GemmParams p = p0;
  p.m_tiles = (p.M + kBM - 1) / kBM;
  p.n_tiles = (p.N + BN - 1) / BN;
  const int units = p.m_tiles * p.n_tiles * p.k_splits;
  const int grid = units < num_sms() ? units : num_sms();
  opt_in_smem<gemm_tcgen05<BN, MX, PEER>>(C::kSmemBytes);
  if (p.ag_flag) {
    // the A rows are guarded by all-gather flags: start while the previous kernel (the
    // add+RMSNorm+all-gather) is still running, as soon as all of its CTAs are resident
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tcgen05<BN, MX, PEER>, ta, tb, p);
    if (e != cudaSuccess) return static_cast<int>(e);
  } else {
    gemm_tcgen05<BN, MX, PEER><<<grid, kGemmThreads, C::kSmemBytes, st>>>(ta, tb, p);
  }
  if (p.k_splits > 1) {
    const int ncols_out = p.epi == kEpiSiluMul ? p.N / 2 : p.N;
    const long threads = static_cast<long>(p.M) * (ncols_out / 8);
    gemm_splitk_reduce<<<static_cast<int>((threads + 255) / 256), 256, 0, st>>>(p);
  }
  return static_cast<int>(cudaGetLastError());
}

// reduce-scatter GEMMs use the instance with the epilogue transpose buffer; every other
// GEMM is built without it
template <int BN, bool MX>
static int launch_bn(const GemmParams& p, const void* A, int lda, const void* B, int ldb, cudaStream_t st) {
  if (p.epi == kEpiPeerRS) return launch_inst<BN, MX, true>(p, A, lda, B, ldb, st);
  return launch_inst<BN, MX, false>(p, A, lda, B, ldb, st);
}

// Waves of a grid of `units` tiles on `sms` SMs.
static double effective_waves(int units, int sms) { return static_cast<double>((units + sms - 1) / sms); }

GemmPlan plan_gemm(int M, int N, int K, int epi, int max_splits) {
  // Pick (BN, k_splits <= max_splits) minimising an estimate of waves x per-unit cost.
  const int sms = num_sms();
  const int kblocks = (K + kBK - 1) / kBK;
  GemmPlan best{256, 1, 1e30};
  const int bns[3] = {256, 128, 64};
  for (int bn : bns) {
    if (epi == kEpiSiluMul && bn < 128) continue;
    const int mt = (M + kBM - 1) / kBM;
    const int nt = (N + bn - 1) / bn;
    for (int ks = 1; ks <= max_splits; ks *= 2) {
      if (ks > 1 && kblocks / ks < 4) break;
      const int units = mt * nt * ks;
      const double waves = effective_waves(units, sms);
      const double kb = static_cast<double>((kblocks + ks - 1) / ks);
      // per unit: MMA time ~ 128*bn*64*2 flop per k-block at ~8.2 TFLOP/s/SM; load time ~ (128+bn)*128 B per
      // k-block at ~40 GB/s/SM (HBM share) -- whichever dominates
      const double t_mma = kb * (128.0 * bn * 64 * 2) / 8.2e12;
      const double t_mem = kb * ((128.0 + bn) * 128) / 43e9;
      double cost = waves * (t_mma > t_mem ? t_mma : t_mem) + 2.5e-6;
      if (ks > 1) cost += (static_cast<double>(ks) * M * N * 4 * 2) / 6.0e12 + 3e-6;  // partial traffic + launch
      if (cost < best.cost * 0.97) best = GemmPlan{bn, ks, cost};
    }
  }
  return best;
}

int gemm_bf16_launch(const GemmParams& p_in, const void* A, int lda, const void* B, int ldb, int bn,
                     cudaStream_t st) {
  GemmParams p = p_in;
  p.k_blocks = (p.K + kBK - 1) / kBK;
  p.kb_per_split = (p.k_blocks + p.k_splits - 1) / p.k_splits;
  p.k_splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  switch (bn) {
    case 256: return launch_bn<256, false>(p, A, lda, B, ldb, st);
    case 128: return launch_bn<128, false>(p, A, lda, B, ldb, st);
    case 64: return launch_bn<64, false>(p, A, lda, B, ldb, st);
    default: return -1;
  }
}

int gemm_grouped_launch(const GemmParams& p_in, const void* A, int lda, int64_t a_rows, const void* B, int ldb,
                        int bn, bool mx, cudaStream_t st) {
  // A: [a_rows, K] expert-sorted activations (segments 128-aligned); B: [G * N, K].
  GemmParams p = p_in;
  if (!p.grp_off || !p.grp_end || p.num_groups < 1 || p.num_groups > kMaxGemmGroups) return -4;
  if (p.k_splits != 1) return -5;
  const int kel = mx ? kBKMx : kBK;
  p.k_blocks = (p.K + kel - 1) / kel;
  p.kb_per_split = p.k_blocks;
  p.M = static_cast<int>(a_rows);                 // tensor-map extent; valid rows come from grp_end
  p.m_tiles = 0;
  // the real tile count is known on the device only: launch one persistent CTA per SM
  const int units_max = static_cast<int>((a_rows + kBM - 1) / kBM) * ((p.N + bn - 1) / bn);
  const int grid = units_max < num_sms() ? (units_max > 0 ? units_max : 1) : num_sms();
  const CUtensorMapDataType dt = mx ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int es = mx ? 1 : 2;
  CUtensorMap ta, tb;
  if (make_tmap_2d(&ta, A, dt, es, a_rows, p.K, lda, kBM, kel)) return -2;
  if (make_tmap_2d(&tb, B, dt, es, static_cast<int64_t>(p.num_groups) * p.N, p.K, ldb, bn, kel)) return -3;
  p.n_tiles = (p.N + bn - 1) / bn;
#define RZ_GROUPED(BNV, MXV)                                                                                   \
  {                                                                                                           \
    using C = GemmCfg<BNV, MXV, false>;                                                                       \
    opt_in_smem<gemm_tcgen05<BNV, MXV, false>>(C::kSmemBytes);                                       \
    gemm_tcgen05<BNV, MXV, false><<<grid, kGemmThreads, C::kSmemBytes, st>>>(ta, tb, p);               \
  }
  if (!mx && bn == 256) RZ_GROUPED(256, false)
  else if (!mx && bn == 128) RZ_GROUPED(128, false)
  else if (mx && bn == 256) RZ_GROUPED(256, true)
  else if (mx && bn == 128) RZ_GROUPED(128, true)
  else return -1;
#undef RZ_GROUPED
  return static_cast<int>(cudaGetLastError());
}

GemmPlan plan_gemm_mxf8(int M, int N, int K, int epi, int max_splits) {
  // Same waves x per-unit cost estimate as the bf16 planner, with the fp8 MMA
  // rate (2x bf16 per SM) and 128-element K blocks.  BN=256 holds a single
  // accumulator (the scale columns take the rest of TMEM), so its epilogue does
  // not overlap the next tile's MMAs: charge it per unit.
  const int sms = num_sms();
  const int kblocks = K / kBKMx;
  GemmPlan best{128, 1, 1e30};
  const int bns[2] = {256, 128};
  // Per unit: MMA time at the measured per-SM rate
  // or tile-load time at ~150 GB/s/SM from L2, whichever dominates, plus a
  // fixed pipeline fill / epilogue cost; the whole GEMM is also bounded below
  // by streaming the weights once from HBM.  Split-K only pays when the tile
  // grid cannot fill half of the SMs (measured: splitting a 1.1-wave grid
  // loses to the fp32 partial traffic).
  const double hbm_floor = (static_cast<double>(N) * K + static_cast<double>(M) * K) / 6.5e12;
  for (int bn : bns) {
    if (N % bn != 0 && bn == 256) continue;
    const int mt = (M + kBM - 1) / kBM;
    const int nt = (N + bn - 1) / bn;
    for (int ks = 1; ks <= max_splits; ks *= 2) {
      if (ks > 1 && (kblocks / ks < 4 || mt * nt * 2 > sms)) break;
      const int units = mt * nt * ks;
      const double waves = effective_waves(units, sms);
      const double kb = static_cast<double>((kblocks + ks - 1) / ks);
      // 128x128 fp8 tiles are shared-memory bound (~10.5 vs ~14 TFLOP/s/SM measured)
      const double t_mma = kb * (128.0 * bn * 128 * 2) / (bn == 256 ? 14e12 : 10.5e12);
      const double t_mem = kb * ((128.0 + bn) * 128 + kSfChunk * (1 + bn / 128)) / 150e9;
      const double t_unit = (t_mma > t_mem ? t_mma : t_mem) + 1.5e-6 + (bn == 256 ? 1.2e-6 : 0.0);
      double cost = waves * t_unit;
      if (cost < hbm_floor) cost = hbm_floor;
      cost += 2.5e-6;
      if (ks > 1) cost += (static_cast<double>(ks) * M * N * 4 * 2) / 6.0e12 + 3e-6;
      if (cost < best.cost * 0.97) best = GemmPlan{bn, ks, cost};
    }
  }
  return best;
}

int gemm_mxf8_launch(const GemmParams& p_in, const void* A, int lda, const void* B, int ldb, int bn,
                     cudaStream_t st) {
  GemmParams p = p_in;
  if (p.K % kBKMx != 0 || p.N % 128 != 0 || !p.sfa || !p.sfb) return -4;
  p.k_blocks = p.K / kBKMx;
  p.kb_per_split = (p.k_blocks + p.k_splits - 1) / p.k_splits;
  p.k_splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  switch (bn) {
    case 256: return launch_bn<256, true>(p, A, lda, B, ldb, st);
    case 128: return launch_bn<128, true>(p, A, lda, B, ldb, st);
    default: return -1;
  }
}

// ---------------------------------------------------------------------------------- MXFP8 quantisation
// 8 threads per (row, 128-column block), 16 elements (two 16-byte loads) per
// thread, 4 blocks per warp; the block's absolute maximum is reduced over its
// 8 lanes.  Rows in [M, M_pad) only get a neutral scale byte (their operand
// rows are zero-filled by the tensor map).
__global__ void __launch_bounds__(256) quant_mxf8_act_kernel(uint8_t* __restrict__ xq, uint8_t* __restrict__ sfa,
                                                             const __nv_bfloat16* __restrict__ x, int M, int M_pad,
                                                             int K, int ldx) {
  const int kblocks = K / 128;
  const long g = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 3;   // (row, block) index
  const int sub = threadIdx.x & 7;
  if (g >= static_cast<long>(M_pad) * kblocks) return;
  const int row = static_cast<int>(g / kblocks);
  const int kb = static_cast<int>(g % kblocks);
  uint8_t* chunk = sfa + (static_cast<size_t>(row / 128) * kblocks + kb) * kSfChunk;
  if (row >= M) {
    if (sub == 0) *reinterpret_cast<uint32_t*>(chunk + sf_offset(row & 127, 0)) = 0x7f7f7f7fu;
    return;
  }
  const __nv_bfloat16* src = x + static_cast<size_t>(row) * ldx + kb * 128 + sub * 16;
  const uint4 u0 = *reinterpret_cast<const uint4*>(src);
  const uint4 u1 = *reinterpret_cast<const uint4*>(src + 8);
  float v[16];
  const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
  const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = __bfloat1622float2(h0[i]), b = __bfloat1622float2(h1[i]);
    v[2 * i] = a.x; v[2 * i + 1] = a.y; v[8 + 2 * i] = b.x; v[8 + 2 * i + 1] = b.y;
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))));
  }
  // the 8 lanes of this (row, block) reduce among themselves; other groups of
  // the warp may have returned (rows past M), so the mask names only this group
  const unsigned gmask = 0xffu << (threadIdx.x & 24);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, o));
  float inv;
  const uint32_t e = ue8m0_scale(amax, &inv);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8x2_storage_t lo =
        __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i] * inv, v[4 * i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi =
        __nv_cvt_float2_to_fp8x2(make_float2(v[4 * i + 2] * inv, v[4 * i + 3] * inv), __NV_SATFINITE, __NV_E4M3);
    w[i] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  *reinterpret_cast<uint4*>(xq + static_cast<size_t>(row) * K + kb * 128 + sub * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  if (sub == 0) *reinterpret_cast<uint32_t*>(chunk + sf_offset(row & 127, 0)) = e * 0x01010101u;
}

int quant_mxf8_act_launch(void* xq, uint8_t* sfa, const __nv_bfloat16* x, int M, int K, int ldx, cudaStream_t st) {
  if (K % 128 != 0) return -1;
  const int M_pad = (M + 127) / 128 * 128;
  const long threads = static_cast<long>(M_pad) * (K / 128) * 8;
  quant_mxf8_act_kernel<<<static_cast<int>((threads + 255) / 256), 256, 0, st>>>(
      static_cast<uint8_t*>(xq), sfa, x, M, M_pad, K, ldx);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz
