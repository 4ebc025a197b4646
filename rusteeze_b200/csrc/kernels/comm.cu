// Peer-memory all-reduce over NVLink 5 / NVSwitch for tensor parallelism.
//
// The reference's collectives are no-ops (crates/rusteeze-engine/src/
// tensor_parallel.rs:80-106).  Here every rank owns a symmetric buffer
// (mapped into all peers' address spaces by torch symmetric memory), laid
// out as [flags | data half 0 | data half 1].  One kernel does the whole
// all-reduce with direct loads/stores to peer memory:
//
//   one-shot (small messages): copy the input into my half, per-block
//     barrier, then each block sums its slice of ALL peers' halves (16-byte
//     P2P loads) into the local output;
//   two-shot (large messages): copy, barrier, block b on rank r reduces
//     sub-chunk b of slice r from every peer and writes it back into its own
//     half, barrier, then gathers sub-chunk b of every slice from its owner.
//
// Every cross-rank dependency stays within one block index (block b on every
// rank touches the same elements), so per-block barriers suffice: block b
// stores the call's epoch into flag[phase][b][my_rank] of every peer with a
// system-scope release, and spins (acquire, bounded by %globaltimer) until
// all peers' flags in its own pad reach the epoch.  The epoch comes from a
// device counter bumped by a 1-thread kernel after each call, so the pair is
// CUDA-graph replayable; the data half alternates with the epoch parity, and
// the first barrier of call e+1 guarantees every rank finished reading call
// e-1's half before anyone overwrites it in call e+1.
// A wait that exceeds 1 s records kCommPeerTimeout in the status word and
// the kernel finishes without blocking (the result is then garbage, and the
// host reports the engine unhealthy).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "comm.h"
#include "common.cuh"

namespace rz {

struct ArParams {
  uint8_t* bufs[kMaxRanks];  // symmetric buffer base of every rank
  const __nv_bfloat16* in;
  __nv_bfloat16* out;
  int64_t n;                 // elements (multiple of 8 * world)
  int64_t half_bytes;        // bytes of one data half
  int rank, world;
  int two_shot;
  uint32_t* epoch_ctr;       // local device counter
  int* status;
};

constexpr int kFlagBytes = 2 * kMaxArBlocks * kMaxRanks * 4;  // [phase][block][rank] uint32

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// block-level barrier across ranks for (phase, blockIdx.x)
__device__ __forceinline__ void peer_barrier(const ArParams& p, int phase, uint32_t epoch) {
  __syncthreads();
  const int t = threadIdx.x;
  if (t < p.world) {
    __threadfence_system();
    uint32_t* flag = reinterpret_cast<uint32_t*>(p.bufs[t]) + (phase * kMaxArBlocks + blockIdx.x) * kMaxRanks + p.rank;
    st_release_sys(flag, epoch);
    const uint32_t* mine =
        reinterpret_cast<const uint32_t*>(p.bufs[p.rank]) + (phase * kMaxArBlocks + blockIdx.x) * kMaxRanks + t;
    if (ld_acquire_sys(mine) < epoch) {
      const uint64_t t0 = globaltimer();
      uint32_t it = 0;
      while (ld_acquire_sys(mine) < epoch) {
        if ((++it & 63u) == 0 && globaltimer() - t0 > kWaitTimeoutNs) {
          set_status(p.status, kCommPeerTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void add8(float* acc, const uint4& u) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float* a) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
  return u;
}

__global__ void __launch_bounds__(512) peer_all_reduce_kernel(ArParams p) {
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.epoch_ctr) + 1u;
  const int64_t half_off = kFlagBytes + static_cast<int64_t>(epoch & 1u) * p.half_bytes;
  const uint4* in = reinterpret_cast<const uint4*>(p.in);
  uint4* out = reinterpret_cast<uint4*>(p.out);
  const int64_t nvec = p.n / 8;
  if (!p.two_shot) {
    uint4* mine = reinterpret_cast<uint4*>(p.bufs[p.rank] + half_off);
    const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
    const int64_t v0 = blockIdx.x * per, v1 = min(nvec, v0 + per);
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) mine[i] = in[i];
    peer_barrier(p, 0, epoch);
    for (int64_t i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int r = 0; r < p.world; ++r) {
        const int rr = (p.rank + r) % p.world;  // stagger the peers each rank reads first
        add8(acc, reinterpret_cast<const uint4*>(p.bufs[rr] + half_off)[i]);
      }
      out[i] = pack8(acc);
    }
    return;
  }
  // two-shot: slice s = [s*nvec/world, (s+1)*nvec/world); block b owns sub-chunk b of every slice
  const int64_t slice = nvec / p.world;
  const int64_t per = (slice + gridDim.x - 1) / gridDim.x;
  const int64_t c0 = blockIdx.x * per, c1 = min(slice, c0 + per);
  uint4* mine = reinterpret_cast<uint4*>(p.bufs[p.rank] + half_off);
  for (int s = 0; s < p.world; ++s)
    for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) mine[s * slice + i] = in[s * slice + i];
  peer_barrier(p, 0, epoch);
  for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int64_t idx = p.rank * slice + i;
    for (int r = 0; r < p.world; ++r) {
      const int rr = (p.rank + r) % p.world;
      add8(acc, reinterpret_cast<const uint4*>(p.bufs[rr] + half_off)[idx]);
    }
    const uint4 v = pack8(acc);
    mine[idx] = v;
    out[idx] = v;
  }
  peer_barrier(p, 1, epoch);
  for (int r = 1; r < p.world; ++r) {
    const int s = (p.rank + r) % p.world;
    const uint4* src = reinterpret_cast<const uint4*>(p.bufs[s] + half_off);
    for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) out[s * slice + i] = src[s * slice + i];
  }
}

__global__ void bump_epoch_kernel(uint32_t* ctr) { *ctr += 1u; }

int peer_all_reduce_launch(const ArParams& p, int blocks, cudaStream_t st) {
  if (p.n == 0) return 0;
  peer_all_reduce_kernel<<<blocks, 512, 0, st>>>(p);
  bump_epoch_kernel<<<1, 1, 0, st>>>(p.epoch_ctr);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace rz

namespace {

// x (local, bf16, numel n) -> out (local) = sum over ranks.  bufs: symmetric buffer bases (one per rank).
int64_t peer_all_reduce(torch::Tensor out, torch::Tensor x, std::vector<int64_t> bufs, int64_t rank,
                        int64_t half_bytes, torch::Tensor epoch, torch::Tensor status, bool two_shot) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && out.is_contiguous(), "contiguous CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "bf16 all-reduce");
  const int world = static_cast<int>(bufs.size());
  TORCH_CHECK(world >= 1 && world <= rz::kMaxRanks, "1..8 ranks");
  const int64_t n = x.numel();
  TORCH_CHECK(n % (8 * world) == 0, "numel must be a multiple of 8 * world");
  TORCH_CHECK(n * 2 <= half_bytes, "message larger than the symmetric buffer half");
  rz::ArParams p{};
  for (int i = 0; i < world; ++i) p.bufs[i] = reinterpret_cast<uint8_t*>(bufs[i]);
  p.in = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.n = n;
  p.half_bytes = half_bytes;
  p.rank = static_cast<int>(rank);
  p.world = world;
  p.two_shot = two_shot ? 1 : 0;
  p.epoch_ctr = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  p.status = status.data_ptr<int>();
  const int64_t vec = n / 8 / (two_shot ? world : 1);
  int blocks = static_cast<int>(std::min<int64_t>(rz::kMaxArBlocks, std::max<int64_t>(1, (vec + 2047) / 2048)));
  const int rc = rz::peer_all_reduce_launch(p, blocks, at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "peer_all_reduce launch failed: ", rc);
  return 2;
}

int64_t flag_bytes() { return rz::kFlagBytes; }

}  // namespace

void bind_comm(pybind11::module_& m) {
  m.def("peer_all_reduce", &peer_all_reduce);
  m.def("peer_flag_bytes", &flag_bytes);
}
