// Allocation-free entry point for split-KV paged decode attention.
// No counterpart in the reference project; see decode_noalloc.h for the
// callers it serves and its contract.
#include "attention.h"
#include "decode_noalloc.h"

#include <atomic>
#include <mutex>

namespace {

// The scratch array and the status word live in the library image: nothing
// is allocated at call time.  Host code must not pass these names to a
// kernel (in host code they denote host-side stand-ins); it passes the device
// addresses looked up below.
static __device__ __align__(256) float g_noalloc_scratch[kRzNoAllocScratchFloats];
static __device__ int g_noalloc_status;

constexpr int kMaxDevices = 64;

struct DeviceSymbols {
  std::atomic<bool> ready{false};
  float* scratch = nullptr;
  int* status = nullptr;
};

// One lookup per device, performed by the first call on that device with it current.
// Host threads making their first call on one device at the same time serialise on the
// mutex; `ready` is published with release ordering after both addresses are written, so
// a thread that sees it set (acquire) also sees the addresses.
int symbols_for_current_device(DeviceSymbols** out) {
  static DeviceSymbols table[kMaxDevices];
  static std::mutex lookup;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kRzNoAllocSymbolError;
  DeviceSymbols& s = table[dev];
  if (!s.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> g(lookup);
    if (!s.ready.load(std::memory_order_relaxed)) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return kRzNoAllocSymbolError;
      void* q = nullptr;
      if (cudaGetSymbolAddress(&q, g_noalloc_status) != cudaSuccess || q == nullptr) return kRzNoAllocSymbolError;
      s.scratch = static_cast<float*>(p);
      s.status = static_cast<int*>(q);
      s.ready.store(true, std::memory_order_release);
    }
  }
  *out = &s;
  return kRzNoAllocOk;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int rz_decode_attention_noalloc(
    __nv_bfloat16* out, int64_t out_stride, const __nv_bfloat16* q, int64_t q_stride, const __nv_bfloat16* k_cache,
    const __nv_bfloat16* v_cache, int64_t block_stride, int num_blocks, const int32_t* seq_lens,
    const int32_t* block_tables, int64_t bt_stride, int num_seqs, int num_q_heads, int num_kv_heads, int head_dim,
    int num_splits, float scale, int window, float softcap, cudaStream_t stream) {
  if (num_seqs <= 0) return kRzNoAllocOk;
  if (!out || !q || !k_cache || !v_cache || !seq_lens || !block_tables || num_splits < 1 || num_kv_heads < 1 ||
      num_q_heads % num_kv_heads != 0)
    return kRzNoAllocBadArgument;
  if (num_splits > 1) {
    const int64_t need = static_cast<int64_t>(num_seqs) * num_q_heads * num_splits * (head_dim + 2);
    if (need > kRzNoAllocScratchFloats) return kRzNoAllocTooLarge;
  }
  DeviceSymbols* sym = nullptr;
  const int rc = symbols_for_current_device(&sym);
  if (rc != kRzNoAllocOk) return rc;
  rz::DecodeAttnParams p{};
  p.out = out;
  p.out_stride = out_stride;
  p.q = q;
  p.q_stride = q_stride;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.block_stride = block_stride;
  p.num_blocks = num_blocks;
  p.seq_lens = seq_lens;
  p.block_tables = block_tables;
  p.bt_stride = bt_stride;
  p.workspace = sym->scratch;
  p.num_seqs = num_seqs;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.num_splits = num_splits;
  p.scale = scale;
  p.window = window;
  p.softcap = softcap;
  p.status = sym->status;
  const int lr = rz::decode_attention_launch(p, stream);
  return lr == -100 ? kRzNoAllocBadArgument : lr;
}

extern "C" __attribute__((visibility("default"))) int rz_decode_attention_noalloc_status(cudaStream_t stream) {
  DeviceSymbols* sym = nullptr;
  if (symbols_for_current_device(&sym) != kRzNoAllocOk) return kRzNoAllocSymbolError;
  int v = 0;
  if (cudaMemcpyAsync(&v, sym->status, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return kRzNoAllocSymbolError;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return kRzNoAllocSymbolError;
  const int zero = 0;
  if (cudaMemcpyAsync(sym->status, &zero, sizeof(int), cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return kRzNoAllocSymbolError;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return kRzNoAllocSymbolError;
  return v;
}
