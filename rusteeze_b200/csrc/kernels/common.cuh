// Shared device helpers for the sm_100a kernels: bf16 math, warp reductions,
// mbarrier / TMA / tcgen05 PTX wrappers, and bounded waits.
//
// Every spin-wait in these kernels is bounded by %globaltimer: after
// kWaitTimeoutNs the waiting thread records an error code in a device status
// word (an int the caller passes in; the host reads it after the step) and
// gives up, so a protocol bug returns an error instead of hanging a shared GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#define RZ_DEVICE __device__ __forceinline__

namespace rz {

// Opts kernel `Kernel` in to at least `bytes` of dynamic shared memory on the current
// device.  The attribute belongs to a device's context, so a process that launches on
// several GPUs (one engine replica per GPU, each on its own thread) needs it once per
// device; and a kernel whose shared memory depends on its arguments (the sampler's row
// slice grows with the vocabulary) must raise it when a larger launch comes: the
// largest size granted per device is recorded, and raising it is serialised so that a
// smaller request can never overwrite a larger grant.
template <auto Kernel>
inline void opt_in_smem(int bytes) {
  static std::atomic<int> granted[64];
  static std::mutex raise;
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (granted[dev].load(std::memory_order_acquire) >= bytes) return;
  std::lock_guard<std::mutex> g(raise);
  if (granted[dev].load(std::memory_order_relaxed) >= bytes) return;
  cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  granted[dev].store(bytes, std::memory_order_release);
}

constexpr uint64_t kWaitTimeoutNs = 1000ull * 1000ull * 1000ull;  // 1 s

enum StatusCode : int {
  kOk = 0,
  kGemmProducerTimeout = 1,
  kGemmMmaTimeout = 2,
  kGemmEpilogueTimeout = 3,
  kCommPeerTimeout = 4,
  kAttnTimeout = 5,
  kBadArgument = 6,
};

// First error wins.
RZ_DEVICE void set_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

RZ_DEVICE uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Race testing of the flag protocols: a pseudo-random pause below max_ns (0: none) keyed by
// (a, b, c), so producers publish in shuffled orders and consumers wait at random points.
RZ_DEVICE void jitter_ns(uint32_t max_ns, uint32_t a, uint32_t b, uint32_t c) {
  if (max_ns == 0) return;
  uint32_t h = a * 0x9E3779B1u ^ (b + 0x7F4A7C15u) * 0x85EBCA77u ^ (c + 0x165667B1u) * 0xC2B2AE3Du;
  h ^= h >> 15;
  h *= 0x2C1B3C6Du;
  h ^= h >> 12;
  __nanosleep(h % max_ns);
}

RZ_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
RZ_DEVICE __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

RZ_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
RZ_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------------ smem / mbarrier
RZ_DEVICE uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

RZ_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
RZ_DEVICE void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
RZ_DEVICE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

RZ_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
RZ_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

RZ_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code` in *status) on timeout.
RZ_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && globaltimer() - t0 > kWaitTimeoutNs) {
      set_status(status, code);
      return false;
    }
  }
}

// ------------------------------------------------------------------ cross-GPU flags (NVLink P2P)
RZ_DEVICE void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
RZ_DEVICE uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Spin until *flag >= target (acquire, system scope), bounded by kWaitTimeoutNs.
RZ_DEVICE bool wait_flag_geq(const uint32_t* flag, uint32_t target, int* status, int code) {
  if (ld_acquire_sys_u32(flag) >= target) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_sys_u32(flag) >= target) return true;
    if ((it & 63u) == 63u && globaltimer() - t0 > kWaitTimeoutNs) {
      set_status(status, code);
      return false;
    }
  }
}
RZ_DEVICE uint32_t ld_relaxed_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
RZ_DEVICE void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Spin until every flag in [flags, flags + n) is >= target.  The flags are polled with
// relaxed loads (independent, so their latencies overlap) and one system-scope fence
// after they are all seen gives the acquire ordering.  Bounded by kWaitTimeoutNs.
// Programmatic dependent launch.  A kernel that calls pdl_trigger() lets the next kernel
// on its stream (launched with the programmatic-serialization attribute) start once
// every CTA of this grid has started; such a dependent synchronises on flags, and calls
// pdl_wait() before it exits so that its completion still implies this grid's.
RZ_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
RZ_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

RZ_DEVICE bool wait_flags_geq(const uint32_t* flags, int n, uint32_t target, int* status, int code) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    bool all = true;
    for (int i = 0; i < n; ++i) all &= ld_relaxed_sys_u32(flags + i) >= target;
    if (all) {
      fence_acq_rel_sys();
      return true;
    }
    if (it == 0) t0 = globaltimer();
    else if ((it & 15u) == 15u && globaltimer() - t0 > kWaitTimeoutNs) {
      set_status(status, code);
      return false;
    }
  }
}

// order generic-proxy writes (peer stores observed through an acquire) before
// later async-proxy (TMA) reads of global memory
RZ_DEVICE void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// barrier among a subset of warps (id != 0; count = threads, a multiple of 32)
RZ_DEVICE void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------------ TMA (no cluster multicast)
RZ_DEVICE void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

RZ_DEVICE void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

RZ_DEVICE void tma_load_4d(void* smem_dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0)
RZ_DEVICE void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ tcgen05
RZ_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
RZ_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// whole warp; writes the TMEM base address to *smem_out
RZ_DEVICE void tmem_alloc(uint32_t* smem_out, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_out)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
RZ_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate)
RZ_DEVICE void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A (M = 128 rows = TMEM lanes) holds two
// bf16 K-elements per 32-bit column, K-ascending from tmem_a
RZ_DEVICE void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f8f6f4 (both operands e4m3), fp32 accumulate
RZ_DEVICE void umma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::mxf8f6f4 with block scaling: e4m3 x e4m3 -> f32, one UE8M0 scale per
// 32 K-elements of every A row and every B row, read from TMEM at tsfa / tsfb
// (the top two address bits select the byte of the 32-bit scale word).
RZ_DEVICE void umma_mxf8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t tsfa,
                         uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// Shared -> tensor memory copy of a 32-row x 16-byte block, replicated into all
// four 32-lane quarters of TMEM (4 columns of 32 bits per lane).
RZ_DEVICE void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Descriptor of a plain (unswizzled) K-major block of 16-byte rows: 8-row core
// matrices 128 bytes apart, a single core matrix along K.
RZ_DEVICE uint64_t smem_desc_rows16(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(128 >> 4) << 32;           // stride byte offset: 8 rows x 16 B
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  return d;                                             // layout type 0: no swizzle
}

// Arrive on an mbarrier when all previously issued tcgen05.mma of this thread complete.
RZ_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns per warp
RZ_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
RZ_DEVICE void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

RZ_DEVICE void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
RZ_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// order this thread's generic-proxy shared-memory writes before later async-proxy
// (tcgen05.mma operand) reads
RZ_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major operand tile stored by TMA with
// 128-byte swizzle (rows of 128 B, 8-row groups 1024 B apart).
RZ_DEVICE uint64_t smem_desc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                  // SWIZZLE_128B
  return d;
}

// Descriptor of an MN-major operand tile stored with 128-byte swizzle: rows of
// 128 B along K (64 bf16 of the M/N dimension each), 8-row groups 1024 B apart
// (stride byte offset), and the next 64 M/N elements `mn_stride` bytes away
// (leading byte offset).
RZ_DEVICE uint64_t smem_desc_mn_sw128(uint32_t saddr, uint32_t mn_stride) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((mn_stride >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}
// Block-scaled kind::mxf8f6f4: e4m3 x e4m3, UE8M0 scales, both K-major.  The
// scale-factor byte ids (which K-chunk of the 32-bit scale word) sit in bits
// 4-5 (B) and 29-30 (A); the accumulator is always f32 in this format.
__host__ __device__ constexpr uint32_t idesc_mxf8(int M, int N, uint32_t sf_id) {
  return (sf_id << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(M >> 4) << 24) | (sf_id << 29);
}
// kind::f8f6f4: e4m3 x e4m3 -> f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace rz
