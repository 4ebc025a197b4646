// Tensor-parallel layer boundary fused with its collectives (NVLink P2P).
//
// Between the row-parallel GEMMs (o_proj, down_proj) and the next column-
// parallel GEMM (QKV, gate/up) the residual stream is sequence-sharded: rank o
// owns rows [o*R, (o+1)*R) (R = rs_rows, a multiple of 8).  The chain is
//
//   GEMM + reduce-scatter   (gemm_tcgen05, kEpiPeerRS): each finished tile row
//                            is stored into its owner's slot for this rank;
//   rs_norm_ag (this file)   the owner sums the world slots of its rows in
//                            fp32, adds its residual shard (kept in bf16 like
//                            the unfused path), RMS-normalises, and stores the
//                            normalised rows into EVERY rank's gather buffer;
//   GEMM on gathered rows    (gemm_tcgen05 with ag_flag): the TMA producer
//                            waits for the all-gather flags of each A tile's
//                            rows before loading it from LOCAL memory.
//
// Synchronisation is by flags carrying an epoch (step counter * 256 + call
// index + 1) stored with st.release.sys and polled with ld.acquire.sys, so no
// flag is ever reset and CUDA-graph replays stay correct; the step counter is
// bumped by `tp_epoch_bump` once per forward.  Buffer reuse needs no extra
// barrier: a rank writes a slot / gather row for call c+1 only after it
// consumed every owner's gather rows of call c, which those owners produced
// after reading their slots of call c.  Every wait is bounded
// (kWaitTimeoutNs); on expiry the status word records kCommPeerTimeout and the
// kernel finishes without blocking.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "common.cuh"
#include "gemm_bf16.h"
#include "mxfp8.cuh"
#include "tp_fused.h"

namespace rz {

__device__ __forceinline__ void ld8f(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8f(const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return u;
}

// 16 warps per block, 2 warps (64 threads) per own row: block b covers rows
// [row0 + 8b, row0 + 8b + 8) (one all-gather flag block) and releases their flag itself.
// Thread t of a row owns the 8-column chunks t, t + 64, ...: CH chunks, kept in registers
// between the sum, the norm and the all-gather so the residual is read once.
constexpr int kRsThreads = 512;

template <int CH, int ROWS = kAgRowBlock>
__global__ void __launch_bounds__(kRsThreads) rs_norm_ag_kernel(RsNormAgParams p) {
  constexpr int kRowThreads = kRsThreads / ROWS;
  constexpr int kRowWarps = kRowThreads / 32;
  // With reduce, this kernel is a programmatic dependent of the reduce-scatter GEMM: its
  // blocks take the SMs that GEMM CTAs leave and finish rows as their m tiles land (every
  // input is flag-guarded; every output is a persistent buffer no earlier kernel reads).
  pdl_trigger();
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(p.epoch_ptr) * 256u + p.call_idx + 1u;
  const int own0 = p.rank * p.rs_rows;
  const int g0 = own0 + blockIdx.x * ROWS;                 // first global row of this block
  if (p.reduce && p.moe_topk > 0) {
    // every (row, slot) of this block was written by the rank that owns the slot's expert
    const int nflags = ROWS * p.moe_topk;
    const int f = threadIdx.x;
    if (f < nflags) {
      const int rr = f / p.moe_topk, k = f % p.moe_topk;
      const int li0 = g0 - own0 + rr;
      if (g0 + rr < p.M && li0 < p.rs_rows)
        wait_flag_geq(p.moe_flag + static_cast<size_t>(k) * p.rs_rows + li0, epoch, p.status, kCommPeerTimeout);
    }
  } else if (p.reduce) {
    // lane quarter (g0 % 128) / 32 of m-tile g0 / 128: both column halves of every n tile,
    // from every source rank (one flag per epilogue warp of the producing GEMM)
    const int mt = g0 / 128, q = (g0 % 128) / 32;
    const int nflags = p.n_tiles * 2 * p.world;
    bool ok = true;
    for (int f = threadIdx.x; f < nflags && ok; f += blockDim.x) {
      const int nt = f / (2 * p.world), h = (f / p.world) & 1, src = f % p.world;
      ok = wait_flag_geq(p.rs_flag + ((static_cast<size_t>(mt) * p.n_tiles + nt) * 8 + q * 2 + h) * p.world + src,
                         epoch, p.status, kCommPeerTimeout);
    }
  }
  __syncthreads();
  static_assert(ROWS == kAgRowBlock, "a CTA holds one whole flag block");
  __shared__ float s_ss[ROWS][kRowWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rr = warp / kRowWarps, sub = warp % kRowWarps;   // row of the block, warp within the row
  const int tr = sub * 32 + lane;                            // thread within the row
  const int row = g0 + rr;                                   // global row
  const int li = row - own0;                                 // row within this rank's shard
  const bool live = row < p.M && li < p.rs_rows;
  uint4 xr[CH];                                              // the rounded residual, bf16
  float ss = 0.f;
  if (live) {
    __nv_bfloat16* res = p.residual + static_cast<size_t>(li) * p.H;
    const int nsrc = p.reduce ? (p.moe_topk > 0 ? p.moe_topk : p.world) : 0;
    // chunks in groups of G with every load of a group issued before the first add, so a
    // thread keeps G (then G per source) 16-byte loads in flight instead of one
    constexpr int G = CH < 4 ? CH : 4;
#pragma unroll
    for (int j0 = 0; j0 < CH; j0 += G) {
      float x[G][8];
      uint4 raw[G];
#pragma unroll
      for (int q = 0; q < G; ++q) {
        const int c = (tr + (j0 + q) * kRowThreads) * 8;
        raw[q] = make_uint4(0u, 0u, 0u, 0u);
        if (c < p.H)
          raw[q] = *reinterpret_cast<const uint4*>(p.reduce ? res + c : p.resid_in + static_cast<size_t>(row) * p.H + c);
      }
#pragma unroll
      for (int q = 0; q < G; ++q) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[q]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          x[q][2 * i] = f.x;
          x[q][2 * i + 1] = f.y;
        }
      }
      for (int s = 0; s < nsrc; ++s) {
        const __nv_bfloat16* slot = p.slots + (static_cast<size_t>(s) * p.rs_rows + li) * p.H;
#pragma unroll
        for (int q = 0; q < G; ++q) {
          const int c = (tr + (j0 + q) * kRowThreads) * 8;
          raw[q] = c < p.H ? *reinterpret_cast<const uint4*>(slot + c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int q = 0; q < G; ++q) {
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[q]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            x[q][2 * i] += f.x;
            x[q][2 * i + 1] += f.y;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < G; ++q) {
        const int j = j0 + q;
        const int c = (tr + j * kRowThreads) * 8;
        if (c < p.H) {
          xr[j] = pack8f(x[q]);
          *reinterpret_cast<uint4*>(res + c) = xr[j];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&xr[j]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {                      // normalise the rounded residual
            const float2 f = __bfloat1622float2(h[i]);
            ss += f.x * f.x + f.y * f.y;
          }
        }
      }
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) s_ss[rr][sub] = ss;
  jitter_ns(p.jitter_ns, epoch, blockIdx.x, static_cast<uint32_t>(warp));
  __syncthreads();
  if (live && p.mx) {
    // MXFP8 rows: the 16 chunks of a 128-column block belong to one half-warp (chunk
    // index tr + 64 j), whose lanes reduce the block maximum together; every lane joins
    // the shuffles (a chunk past H contributes 0)
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kRowWarps; ++i) tot += s_ss[rr][i];
    const float inv = rsqrtf(tot / p.H + p.eps);
    const int kbo = p.H / 128;
    const size_t sf_row = static_cast<size_t>(row / 128) * kbo;
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = (tr + j * kRowThreads) * 8;
      const bool ok = c < p.H;
      float x[8], w[8];
      float amax = 0.f;
      if (ok) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&xr[j]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          x[2 * i] = f.x;
          x[2 * i + 1] = f.y;
        }
        ld8f(p.w + c, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          x[i] = x[i] * inv * (w[i] + p.offset);          // quantised from fp32, as rms_norm_mxf8 does
          amax = fmaxf(amax, fabsf(x[i]));
        }
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (ok) {
        float qinv;
        const uint32_t e = ue8m0_scale(amax, &qinv);
        const uint2 q = pack_e4m3x8(x, qinv);
        const int kb = c / 128;
        for (int d = 0; d < p.world; ++d) {
          *reinterpret_cast<uint2*>(p.gather_q[d] + static_cast<size_t>(row) * p.H + c) = q;
          if ((tr & 15) == 0)
            *reinterpret_cast<uint32_t*>(p.gather_sf[d] + (sf_row + kb) * kSfChunkBytes + sf_offset(row & 127, 0)) =
                e * 0x01010101u;
        }
      }
    }
  } else if (live) {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kRowWarps; ++i) tot += s_ss[rr][i];
    const float inv = rsqrtf(tot / p.H + p.eps);
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = (tr + j * kRowThreads) * 8;
      if (c < p.H) {
        float x[8], w[8];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&xr[j]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h[i]);
          x[2 * i] = f.x;
          x[2 * i + 1] = f.y;
        }
        ld8f(p.w + c, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = x[i] * inv * (w[i] + p.offset);
        const uint4 o = pack8f(x);
        for (int d = 0; d < p.world; ++d)
          *reinterpret_cast<uint4*>(p.gather[d] + static_cast<size_t>(row) * p.H + c) = o;
      }
    }
  }
  // publish: the block barrier orders every thread's stores before the flag thread's
  // system-scope fence + release (cumulative), so one fence per destination suffices
  __syncthreads();
  if (threadIdx.x < p.world && g0 < p.M) {
    jitter_ns(p.jitter_ns, epoch + 1u, blockIdx.x, threadIdx.x);
    __threadfence_system();
    st_release_sys_u32(p.ag_flag[threadIdx.x] + g0 / kAgRowBlock, epoch);
  }
  pdl_wait();   // complete only after the primary grid
}

__global__ void tp_epoch_bump_kernel(uint32_t* ep) { *ep += 1u; }

// One warp per group of 8 consecutive (token, slot) pairs: the warp stores the group's
// weighted rows, then one lane fences once (system scope) and releases the group's flags.
// A fence per row made the kernel fence-bound (membar stalls dominated); the owner still
// waits per (row, slot) flag.
constexpr int kMoePairsPerWarp = 8;
__global__ void __launch_bounds__(256) moe_combine_peer_kernel(MoeCombinePeerParams p) {
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(p.epoch_ptr) * 256u + p.call_idx + 1u;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int pairs = p.M * p.topk;
  const int groups = (pairs + kMoePairsPerWarp - 1) / kMoePairsPerWarp;
  for (int gi = blockIdx.x * warps + (threadIdx.x >> 5); gi < groups; gi += gridDim.x * warps) {
    const int i0 = gi * kMoePairsPerWarp;
    const int i1 = min(pairs, i0 + kMoePairsPerWarp);
    bool any = false;
    for (int i = i0; i < i1; ++i) {
      const int pos = p.pos_of[i];
      if (pos < 0) continue;                                 // warp-uniform: the expert is on another rank
      any = true;
      const int t = i / p.topk, k = i % p.topk;
      const int owner = t / p.rs_rows, li = t - owner * p.rs_rows;
      const float w = p.topk_w[i];
      const __nv_bfloat16* src = p.y + static_cast<size_t>(pos) * p.H;
      __nv_bfloat16* dst = p.slot[owner] + (static_cast<size_t>(k) * p.rs_rows + li) * p.H;
      for (int c = lane * 8; c < p.H; c += 256) {
        float v[8];
        ld8f(src + c, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] *= w;
        *reinterpret_cast<uint4*>(dst + c) = pack8f(v);
      }
    }
    __syncwarp();
    if (lane == 0 && any) {
      jitter_ns(p.jitter_ns, epoch, static_cast<uint32_t>(gi), blockIdx.x);
      __threadfence_system();      // orders the whole warp's row stores (after the warp barrier)
      for (int i = i0; i < i1; ++i) {
        if (p.pos_of[i] < 0) continue;
        const int t = i / p.topk, k = i % p.topk;
        const int owner = t / p.rs_rows, li = t - owner * p.rs_rows;
        st_release_sys_u32(p.flag[owner] + static_cast<size_t>(k) * p.rs_rows + li, epoch);
      }
    }
  }
}

__global__ void ag_wait_kernel(const uint32_t* ag_flag, int nrb, const uint32_t* epoch_ptr, uint32_t call_idx,
                               int* status) {
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(epoch_ptr) * 256u + call_idx + 1u;
  for (int rb = blockIdx.x * blockDim.x + threadIdx.x; rb < nrb; rb += gridDim.x * blockDim.x)
    if (!wait_flag_geq(ag_flag + rb, epoch, status, kCommPeerTimeout)) return;
}

int moe_combine_peer_launch(const MoeCombinePeerParams& p, cudaStream_t st) {
  if (p.H % 8 != 0) return -1;
  const int pairs = p.M * p.topk;
  if (pairs == 0) return 0;
  const int groups = (pairs + kMoePairsPerWarp - 1) / kMoePairsPerWarp;
  int blocks = (groups + 7) / 8;
  blocks = blocks > 1024 ? 1024 : blocks;
  moe_combine_peer_kernel<<<blocks, 256, 0, st>>>(p);
  return static_cast<int>(cudaGetLastError());
}

int ag_wait_launch(const uint32_t* ag_flag, int M, const uint32_t* epoch_ptr, uint32_t call_idx, int* status,
                   cudaStream_t st) {
  const int nrb = (M + kAgRowBlock - 1) / kAgRowBlock;
  if (nrb == 0) return 0;
  ag_wait_kernel<<<(nrb + 127) / 128, 128, 0, st>>>(ag_flag, nrb, epoch_ptr, call_idx, status);
  return static_cast<int>(cudaGetLastError());
}


int rs_norm_ag_launch(const RsNormAgParams& p, cudaStream_t st) {
  if (p.rs_rows % kAgRowBlock != 0 || p.H % 8 != 0 || p.H > kRsNormAgMaxH || p.world > kMaxTpRanks ||
      kAgRowBlock * p.moe_topk > kRsThreads || (p.mx && p.H % 128 != 0))
    return -1;
  const int own = min(p.M, (p.rank + 1) * p.rs_rows) - p.rank * p.rs_rows;
  if (own <= 0) return 0;
  const int ch = (p.H / 8 + kRsThreads / kAgRowBlock - 1) / (kRsThreads / kAgRowBlock);
  void (*k)(RsNormAgParams) = ch <= 4    ? rs_norm_ag_kernel<4>
                              : ch <= 8  ? rs_norm_ag_kernel<8>
                              : ch <= 12 ? rs_norm_ag_kernel<12>
                                         : rs_norm_ag_kernel<16>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((own + kAgRowBlock - 1) / kAgRowBlock);
  cfg.blockDim = dim3(kRsThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.reduce ? 1 : 0;     // the replicated input of reduce == 0 is not flag-guarded
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaGetLastError());
}

int tp_epoch_bump_launch(uint32_t* ep, cudaStream_t st) {
  tp_epoch_bump_kernel<<<1, 1, 0, st>>>(ep);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz
