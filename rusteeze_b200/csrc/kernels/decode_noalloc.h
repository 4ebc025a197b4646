// Allocation-free entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that cannot allocate device memory at call time.
// Examples: an application whose device memory is entirely owned by its own
// pool or by another runtime (so an extra cudaMalloc would fail or break its
// accounting), or a latency-critical loop that must not hit cudaMalloc/cudaFree,
// which can synchronise the device.  The regular entry point (the torch op
// `decode_attention`) takes a caller-provided workspace; this one uses a fixed
// buffer that is part of the library image instead.
//
// Scratch: a file-scope `static __device__` array of kRzNoAllocScratchFloats
// fp32 values (16 MiB) holding the split-KV partial results.  Every GPU that
// loads this library keeps that array resident until the process exits.
//
// Contract:
//   * Inputs and outputs are the caller's device pointers, laid out as for
//     the regular entry point (q rows [num_seqs, Hq, D] with row stride
//     q_stride; out rows with row stride out_stride; per-layer cache view
//     [num_blocks, Hkv, 16, D] with block_stride elements between blocks;
//     int32 seq_lens [num_seqs] and block tables [num_seqs, bt_stride]).
//   * It calls no cudaMalloc / cudaFree and no allocating library routine.
//   * The first call on each device looks up the device address of the
//     scratch array (cudaGetSymbolAddress) with that device current; make
//     that first call before any stream capture.
//   * All calls share the one scratch array, which keeps the previous call's
//     contents.  Nothing in it has to start at zero: every partial a call
//     reads was written earlier by the same call.  Calls that overlap on the
//     GPU (different streams, or different host threads on one device) race
//     on the array; serialise them.
//   * Sizes whose partials do not fit (num_seqs * num_q_heads * num_splits *
//     (head_dim + 2) > kRzNoAllocScratchFloats when num_splits > 1) are
//     rejected with kRzNoAllocTooLarge before anything is launched.
//   * A bad page id or sequence length found by the kernel's bounds checks is
//     recorded in a device status word; rz_decode_attention_noalloc_status()
//     copies it to the host and clears it.  Like the scratch array, the status
//     word is one per device and shared by every call on it: a code it reports
//     may come from any call since the last read, including an overlapping one.
//     If clearing it fails, kRzNoAllocSymbolError is returned instead of the
//     code, so a stale code is not reported again as new.
//   * The per-device address lookup is safe to run from several host threads
//     at once (it is serialised); the calls themselves still race on the GPU
//     as described above.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define kRzNoAllocScratchFloats (4 * 1024 * 1024)

enum {
  kRzNoAllocOk = 0,
  kRzNoAllocTooLarge = -201,       // partials exceed the static scratch
  kRzNoAllocBadArgument = -202,    // unsupported head_dim / group size, null pointers
  kRzNoAllocSymbolError = -203,    // cudaGetSymbolAddress failed on this device
};

// Returns 0 on success, a kRzNoAlloc* code, or a positive cudaError_t from the launch.
int rz_decode_attention_noalloc(__nv_bfloat16* out, int64_t out_stride, const __nv_bfloat16* q, int64_t q_stride,
                                const __nv_bfloat16* k_cache, const __nv_bfloat16* v_cache, int64_t block_stride,
                                int num_blocks, const int32_t* seq_lens, const int32_t* block_tables,
                                int64_t bt_stride, int num_seqs, int num_q_heads, int num_kv_heads, int head_dim,
                                int num_splits, float scale, int window, float softcap, cudaStream_t stream);

// Reads (and clears) the device status word of the allocation-free path; synchronises `stream`.
int rz_decode_attention_noalloc_status(cudaStream_t stream);

#ifdef __cplusplus
}
#endif
