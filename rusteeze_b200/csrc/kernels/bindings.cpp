// torch bindings for the sm_100a kernels.  Each op validates shapes/dtypes,
// launches on the current CUDA stream, and raises on a launch error.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <torch/extension.h>

#include "attention.h"
#include "elementwise.h"
#include "gemm_bf16.h"
#include "gemm_fp8.h"
#include "moe.h"
#include "tp_fused.h"
#include "sampling.h"
#include "comm.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")
#define CHECK_LAST(x) TORCH_CHECK((x).stride(-1) == 1, #x " must be contiguous in the last dim")

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

inline void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed with code ", rc, " (", (rc > 0 ? cudaGetErrorString(static_cast<cudaError_t>(rc)) : "bad argument"), ")");
}

// One status word per device for the bounded device-side waits.
// Created on first use under a lock: replicas on several host threads may make their
// first launches at the same time.
torch::Tensor& status_tensor(int dev) {
  static torch::Tensor t[64];
  static std::mutex init;
  std::lock_guard<std::mutex> g(init);
  if (!t[dev].defined())
    t[dev] = torch::zeros({4}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev));
  return t[dev];
}
int* status_ptr() {
  int dev;
  cudaGetDevice(&dev);
  return status_tensor(dev).data_ptr<int>();
}

void rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor w, double eps, double offset) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w);
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "rms_norm: contiguous tensors required");
  const int H = x.size(-1);
  const int rows = x.numel() / H;
  check_rc(rz::rms_norm_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                               reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), nullptr,
                               reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rows, H, eps, offset,
                               cur_stream()),
           "rms_norm");
}

void fused_add_rms_norm(torch::Tensor out, torch::Tensor x, torch::Tensor residual, torch::Tensor w, double eps,
                        double offset) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(residual); CHECK_BF16(w);
  TORCH_CHECK(x.is_contiguous() && residual.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
  const int H = x.size(-1);
  const int rows = x.numel() / H;
  check_rc(rz::rms_norm_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                               reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                               reinterpret_cast<__nv_bfloat16*>(residual.data_ptr()),
                               reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rows, H, eps, offset,
                               cur_stream()),
           "fused_add_rms_norm");
}

// KV cache element format from the cache tensor's dtype: bf16, or fp8 e4m3 / e5m2
static int kv_format(const torch::Tensor& c) {
  switch (c.scalar_type()) {
    case at::kBFloat16: return rz::kKvBf16;
    case at::kFloat8_e4m3fn: return rz::kKvE4m3;
    case at::kFloat8_e5m2: return rz::kKvE5m2;
    default: TORCH_CHECK(false, "KV cache must be bfloat16, float8_e4m3fn or float8_e5m2");
  }
  return -1;
}

void rope_and_cache(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin, torch::Tensor k_cache,
                    torch::Tensor v_cache, torch::Tensor slots, int64_t Hq, int64_t Hkv, int64_t D, double k_scale,
                    double v_scale) {
  const at::cuda::CUDAGuard rz_guard(qkv.device());
  CHECK_CUDA(qkv); CHECK_BF16(qkv); CHECK_LAST(qkv);
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong, "int64 positions/slots");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "fp32 contiguous cos_sin");
  TORCH_CHECK(k_cache.stride(0) == v_cache.stride(0), "k/v caches must share the block stride");
  TORCH_CHECK(k_cache.stride(1) == 16 * D && k_cache.stride(2) == D, "cache page layout [blocks, Hkv, 16, D]");
  const int fmt = kv_format(k_cache);
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "k/v caches must share the dtype");
  TORCH_CHECK(k_scale > 0 && v_scale > 0, "KV cache scales must be positive");
  check_rc(rz::rope_cache_launch(reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0),
                                 positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(), k_cache.data_ptr(),
                                 v_cache.data_ptr(), k_cache.stride(0), slots.data_ptr<int64_t>(), qkv.size(0), Hq,
                                 Hkv, D, fmt, static_cast<float>(k_scale), static_cast<float>(v_scale),
                                 cur_stream()),
           "rope_and_cache");
}

// fp8 cache blocks of sequences [seq_offset, seq_offset + num_seqs) -> bf16 scratch pages and
// the scratch block table (rows indexed like block_tables)
void kv_dequant_gather(torch::Tensor k_out, torch::Tensor v_out, torch::Tensor bt_out, torch::Tensor k_cache,
                       torch::Tensor v_cache, torch::Tensor block_tables, torch::Tensor seq_lens, int64_t seq_offset,
                       int64_t num_seqs, double k_scale, double v_scale) {
  const at::cuda::CUDAGuard rz_guard(k_out.device());
  CHECK_CUDA(k_out); CHECK_BF16(k_out); CHECK_BF16(v_out);
  TORCH_CHECK(k_out.is_contiguous() && v_out.is_contiguous() && k_out.sizes() == v_out.sizes(),
              "scratch pages [blocks, Hkv, 16, D], contiguous");
  TORCH_CHECK(bt_out.scalar_type() == at::kInt && bt_out.stride(1) == 1, "int32 scratch block table");
  TORCH_CHECK(bt_out.size(0) >= seq_offset + num_seqs, "scratch block table has too few rows");
  const int fmt = kv_format(k_cache);
  TORCH_CHECK(fmt != rz::kKvBf16 && v_cache.scalar_type() == k_cache.scalar_type(), "fp8 k/v caches");
  TORCH_CHECK(k_cache.stride(0) == v_cache.stride(0) && k_cache.size(1) == k_out.size(1) &&
                  k_cache.size(3) == k_out.size(3) && k_cache.stride(1) == 16 * k_cache.size(3),
              "cache and scratch page layouts differ");
  check_rc(rz::kv_dequant_gather_launch(
               reinterpret_cast<__nv_bfloat16*>(k_out.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_out.data_ptr()),
               bt_out.data_ptr<int32_t>(), bt_out.stride(0), reinterpret_cast<const uint8_t*>(k_cache.data_ptr()),
               reinterpret_cast<const uint8_t*>(v_cache.data_ptr()), k_cache.stride(0), k_cache.size(0),
               block_tables.data_ptr<int32_t>(), block_tables.stride(0), seq_lens.data_ptr<int32_t>(), seq_offset,
               num_seqs, k_cache.size(1), k_cache.size(3), fmt, static_cast<float>(k_scale),
               static_cast<float>(v_scale), k_out.size(0), status_ptr(), cur_stream()),
           "kv_dequant_gather");
}

// Vocab-parallel embedding rows: table holds rows [lo, hi) of the vocabulary.
void embedding(torch::Tensor out, torch::Tensor table, torch::Tensor ids, int64_t lo, int64_t hi, int64_t vocab,
               double scale) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(table); CHECK_BF16(table); CHECK_LAST(table);
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "embedding: int64 ids");
  TORCH_CHECK(out.is_contiguous() && out.size(1) == table.size(1) && out.size(0) == ids.numel(), "embedding: out [M, H]");
  TORCH_CHECK(table.stride(0) == table.size(1), "embedding: contiguous table rows");
  check_rc(rz::embedding_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), ids.data_ptr<int64_t>(),
                                static_cast<int>(ids.numel()), static_cast<int>(table.size(1)), lo, hi, vocab,
                                static_cast<float>(scale), status_ptr(), cur_stream()),
           "embedding");
}

void layer_norm(torch::Tensor out, torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w,
                c10::optional<torch::Tensor> b, double eps) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w);
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "layer_norm: contiguous rows");
  const int rows = x.size(0), H = x.size(1);
  check_rc(rz::layer_norm_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                 reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                 residual.has_value() ? reinterpret_cast<__nv_bfloat16*>(residual->data_ptr()) : nullptr,
                                 reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                                 b.has_value() ? reinterpret_cast<const __nv_bfloat16*>(b->data_ptr()) : nullptr, rows, H,
                                 static_cast<float>(eps), cur_stream()),
           "layer_norm");
}

void act_mul(torch::Tensor out, torch::Tensor x, int64_t kind) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(x); CHECK_BF16(x);
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
  check_rc(rz::act_mul_launch(reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                              reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.size(0), x.size(1) / 2, kind,
                              cur_stream()),
           "act_mul");
}

// ALiBi slopes: fp32 on the device, one per query head of this rank
static const float* alibi_ptr(const c10::optional<torch::Tensor>& a, int64_t heads) {
  if (!a.has_value()) return nullptr;
  CHECK_CUDA(*a);
  TORCH_CHECK(a->scalar_type() == at::kFloat && a->is_contiguous() && a->numel() == heads,
              "alibi slopes must be a contiguous fp32 tensor with one slope per query head");
  return a->data_ptr<float>();
}

void decode_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                      torch::Tensor seq_lens, torch::Tensor block_tables, c10::optional<torch::Tensor> workspace,
                      int64_t num_seqs, double scale, int64_t window, double softcap, int64_t num_splits,
                      c10::optional<torch::Tensor> alibi, double k_scale, double v_scale) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(q); CHECK_BF16(q);
  rz::DecodeAttnParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_stride = out.stride(0);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.q_stride = q.stride(0);
  TORCH_CHECK(q.stride(1) == q.size(2) && q.stride(2) == 1, "q rows must hold [Hq, D] contiguously");
  p.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  p.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  p.block_stride = k_cache.stride(0);
  p.num_blocks = k_cache.size(0);
  p.seq_lens = seq_lens.data_ptr<int32_t>();
  p.block_tables = block_tables.data_ptr<int32_t>();
  p.bt_stride = block_tables.stride(0);
  p.num_seqs = num_seqs;
  p.num_q_heads = q.size(1);
  p.num_kv_heads = k_cache.size(1);
  p.head_dim = q.size(2);
  p.num_splits = num_splits;
  p.scale = scale;
  p.window = window;
  p.softcap = softcap;
  p.alibi = alibi_ptr(alibi, p.num_q_heads);
  p.kv_fmt = kv_format(k_cache);
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "k/v caches must share the dtype");
  TORCH_CHECK(k_scale > 0 && v_scale > 0, "KV cache scales must be positive");
  p.k_scale = static_cast<float>(k_scale);
  p.v_scale = static_cast<float>(v_scale);
  p.status = status_ptr();
  if (num_splits > 1) {
    TORCH_CHECK(workspace.has_value() &&
                    workspace->numel() >= num_seqs * p.num_q_heads * num_splits * (p.head_dim + 2),
                "decode workspace too small");
    p.workspace = workspace->data_ptr<float>();
  }
  check_rc(rz::decode_attention_launch(p, cur_stream()), "decode_attention");
}

void prefill_attention_impl(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor qsl, torch::Tensor seq_lens, torch::Tensor block_tables, int64_t seq_offset,
                            int64_t num_seqs, int64_t max_q_len, double scale, int64_t window, double softcap,
                            int64_t impl, c10::optional<torch::Tensor> alibi) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(q); CHECK_BF16(q);
  rz::PrefillAttnParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_stride = out.stride(0);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.q_stride = q.stride(0);
  p.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  p.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  p.block_stride = k_cache.stride(0);
  p.num_blocks = k_cache.size(0);
  p.query_start_loc = qsl.data_ptr<int32_t>();
  p.seq_lens = seq_lens.data_ptr<int32_t>();
  p.block_tables = block_tables.data_ptr<int32_t>();
  p.bt_stride = block_tables.stride(0);
  p.seq_offset = seq_offset;
  p.num_seqs = num_seqs;
  p.max_q_len = max_q_len;
  p.num_q_heads = q.size(1);
  p.num_kv_heads = k_cache.size(1);
  p.head_dim = q.size(2);
  p.scale = scale;
  p.window = window;
  p.softcap = softcap;
  p.alibi = alibi_ptr(alibi, p.num_q_heads);
  TORCH_CHECK(k_cache.scalar_type() == at::kBFloat16 && v_cache.scalar_type() == at::kBFloat16,
              "prefill attention reads bf16 pages (gather an fp8 cache with kv_dequant_gather first)");
  p.status = status_ptr();
  // impl: 0 = tensor-core kernel when the shape allows it (head_dim 128), else mma.sync;
  //       1 = mma.sync kernel; 2 = tensor-core kernel (error if the shape is not supported)
  const bool tc = impl != 1 && rz::prefill_tc_supported(p);
  TORCH_CHECK(impl != 2 || tc, "prefill_attention: shape not supported by the tcgen05 kernel");
  check_rc(tc ? rz::prefill_tc_launch(p, cur_stream()) : rz::prefill_attention_launch(p, cur_stream()),
           "prefill_attention");
}

void prefill_attention(torch::Tensor out, torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                       torch::Tensor qsl, torch::Tensor seq_lens, torch::Tensor block_tables, int64_t seq_offset,
                       int64_t num_seqs, int64_t max_q_len, double scale, int64_t window, double softcap,
                       c10::optional<torch::Tensor> alibi) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  prefill_attention_impl(out, q, k_cache, v_cache, qsl, seq_lens, block_tables, seq_offset, num_seqs, max_q_len,
                         scale, window, softcap, 0, alibi);
}

// ---------------------------------------------------------------- GEMM

std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t epi) {
  auto pl = rz::plan_gemm(M, N, K, epi);
  return {pl.bn, pl.k_splits};
}

// Returns the number of kernels launched (1, or 2 with a split-K reduction).
int64_t gemm_bf16_ex(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                     c10::optional<torch::Tensor> residual, int64_t epi, int64_t bn, int64_t k_splits) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w); CHECK_LAST(x); CHECK_LAST(w);
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm: K mismatch");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "gemm: K and N must be multiples of 8");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "gemm: row strides must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "gemm: operands must be 16-byte aligned");
  if ((epi & 0xff) == rz::kEpiSiluMul) TORCH_CHECK(N % 128 == 0 && out.size(1) == N / 2, "silu epilogue: N % 128, out N/2");
  if (bn <= 0 || k_splits <= 0) {
    auto pl = rz::plan_gemm(M, N, K, static_cast<int>(epi & 0xff));
    bn = pl.bn;
    k_splits = pl.k_splits;
  }
  rz::GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.k_splits = k_splits;
  p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldd = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.residual = residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  p.ldr = residual.has_value() ? residual->stride(0) : 0;
  p.epi = static_cast<int>(epi & 0xff);
  p.gate_act = static_cast<int>((epi >> 8) & 1);   // kGateGelu: GELU(tanh) gate
  p.status = status_ptr();
  torch::Tensor ws;
  if (k_splits > 1) {
    ws = torch::empty({k_splits, M, N}, x.options().dtype(torch::kFloat32));
    p.partial = ws.data_ptr<float>();
  }
  check_rc(rz::gemm_bf16_launch(p, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), bn, cur_stream()),
           "gemm_bf16");
  return k_splits > 1 ? 2 : 1;
}

int64_t gemm_bf16(torch::Tensor out, torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                  c10::optional<torch::Tensor> residual) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  return gemm_bf16_ex(out, x, w, bias, residual, 0, 0, 0);
}

// ---------------------------------------------------------------- FP8
void quant_fp8_act(torch::Tensor xq, torch::Tensor xs, torch::Tensor x) {
  const at::cuda::CUDAGuard rz_guard(xq.device());
  CHECK_CUDA(x); CHECK_BF16(x);
  TORCH_CHECK(x.size(1) % 128 == 0, "K must be a multiple of 128");
  check_rc(rz::quant_fp8_act_launch(xq.data_ptr(), xs.data_ptr<float>(),
                                    reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.size(0), x.size(1),
                                    x.stride(0), xs.stride(0), cur_stream()),
           "quant_fp8_act");
}

// Returns the number of kernels launched.
int64_t gemm_fp8_block(torch::Tensor out, torch::Tensor xq, torch::Tensor xs, torch::Tensor wq, torch::Tensor ws,
                       c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> residual, int64_t epi,
                       int64_t k_splits) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  const int M = xq.size(0), K = xq.size(1), N = wq.size(0);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "fp8 gemm: K and N must be multiples of 128");
  TORCH_CHECK(wq.size(1) == K, "fp8 gemm: K mismatch");
  TORCH_CHECK(xq.element_size() == 1 && wq.element_size() == 1, "fp8 gemm: e4m3 operands");
  TORCH_CHECK(xs.scalar_type() == at::kFloat && ws.scalar_type() == at::kFloat, "fp8 gemm: fp32 scales");
  if (epi == rz::kEpiSiluMul) TORCH_CHECK(out.size(1) == N / 2, "silu epilogue: out has N/2 columns");
  if (k_splits <= 0) k_splits = rz::fp8_plan_splits(M, N, K);
  rz::Fp8GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.k_splits = k_splits;
  p.epi = epi;
  p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldd = out.stride(0);
  p.a_scale = xs.data_ptr<float>();
  p.a_scale_ld = xs.stride(0);
  p.b_scale = ws.data_ptr<float>();
  p.b_scale_ld = ws.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.residual = residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  p.ldr = residual.has_value() ? residual->stride(0) : 0;
  p.status = status_ptr();
  torch::Tensor wsp;
  if (k_splits > 1) {
    wsp = torch::empty({k_splits, M, N}, xq.options().dtype(torch::kFloat32));
    p.partial = wsp.data_ptr<float>();
  }
  check_rc(rz::gemm_fp8_launch(p, xq.data_ptr(), xq.stride(0), wq.data_ptr(), wq.stride(0), cur_stream()),
           "gemm_fp8_block");
  return k_splits > 1 ? 2 : 1;
}

// ---------------------------------------------------------------- MXFP8 (UE8M0 block scales)
void quant_mxf8_act(torch::Tensor xq, torch::Tensor sfa, torch::Tensor x) {
  const at::cuda::CUDAGuard rz_guard(xq.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_LAST(x);
  const int M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "K must be a multiple of 128");
  TORCH_CHECK(xq.is_contiguous() && xq.size(0) == M && xq.size(1) == K && xq.element_size() == 1, "xq: e4m3 [M, K]");
  TORCH_CHECK(sfa.is_contiguous() && sfa.numel() >= static_cast<int64_t>((M + 127) / 128) * (K / 128) * 512,
              "sfa: ceil(M/128) * K/128 chunks of 512 bytes");
  check_rc(rz::quant_mxf8_act_launch(xq.data_ptr(), reinterpret_cast<uint8_t*>(sfa.data_ptr()),
                                     reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), M, K, x.stride(0),
                                     cur_stream()),
           "quant_mxf8_act");
}

void rms_norm_mxf8(torch::Tensor xq, torch::Tensor sfa, torch::Tensor x, c10::optional<torch::Tensor> residual,
                   torch::Tensor w, double eps, double offset) {
  const at::cuda::CUDAGuard rz_guard(xq.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w);
  TORCH_CHECK(x.is_contiguous() && xq.is_contiguous() && sfa.is_contiguous(), "rms_norm_mxf8: contiguous tensors");
  const int M = x.size(0), H = x.size(1);
  TORCH_CHECK(xq.size(0) == M && xq.size(1) == H && xq.element_size() == 1, "xq: e4m3 [M, H]");
  TORCH_CHECK(sfa.numel() >= static_cast<int64_t>((M + 127) / 128) * (H / 128) * 512, "sfa too small");
  __nv_bfloat16* res = nullptr;
  if (residual.has_value()) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == x.sizes(), "residual [M, H]");
    res = reinterpret_cast<__nv_bfloat16*>(residual->data_ptr());
  }
  check_rc(rz::rms_norm_mxf8_launch(reinterpret_cast<uint8_t*>(xq.data_ptr()), reinterpret_cast<uint8_t*>(sfa.data_ptr()),
                                    reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), res,
                                    reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), M, H, eps, offset,
                                    cur_stream()),
           "rms_norm_mxf8");
}

// Returns the number of kernels launched (1, or 2 with a split-K reduction).
int64_t gemm_mxf8(torch::Tensor out, torch::Tensor xq, torch::Tensor sfa, torch::Tensor wq, torch::Tensor sfb,
                  c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> residual, int64_t epi, int64_t bn,
                  int64_t k_splits) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(xq);
  const int M = xq.size(0), K = xq.size(1), N = wq.size(0);
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0, "mxf8 gemm: K and N must be multiples of 128");
  TORCH_CHECK(wq.size(1) == K && xq.is_contiguous() && wq.is_contiguous(), "mxf8 gemm: contiguous [M,K] x [N,K]");
  TORCH_CHECK(xq.element_size() == 1 && wq.element_size() == 1, "mxf8 gemm: e4m3 operands");
  TORCH_CHECK(sfa.numel() >= static_cast<int64_t>((M + 127) / 128) * (K / 128) * 512 &&
                  sfb.numel() >= static_cast<int64_t>(N / 128) * (K / 128) * 512,
              "mxf8 gemm: scale chunk buffers too small");
  if ((epi & 0xff) == rz::kEpiSiluMul) TORCH_CHECK(out.size(1) == N / 2, "silu epilogue: out has N/2 columns");
  if (bn <= 0 || k_splits <= 0) {
    auto pl = rz::plan_gemm_mxf8(M, N, K, static_cast<int>(epi & 0xff));
    bn = pl.bn;
    k_splits = pl.k_splits;
  }
  rz::GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.k_splits = k_splits;
  p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldd = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.residual = residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  p.ldr = residual.has_value() ? residual->stride(0) : 0;
  p.epi = static_cast<int>(epi & 0xff);
  p.gate_act = static_cast<int>((epi >> 8) & 1);   // kGateGelu: GELU(tanh) gate
  p.status = status_ptr();
  p.sfa = reinterpret_cast<const uint8_t*>(sfa.data_ptr());
  p.sfb = reinterpret_cast<const uint8_t*>(sfb.data_ptr());
  torch::Tensor ws;
  if (k_splits > 1) {
    ws = torch::empty({k_splits, M, N}, xq.options().dtype(torch::kFloat32));
    p.partial = ws.data_ptr<float>();
  }
  check_rc(rz::gemm_mxf8_launch(p, xq.data_ptr(), xq.stride(0), wq.data_ptr(), wq.stride(0), bn, cur_stream()),
           "gemm_mxf8");
  return k_splits > 1 ? 2 : 1;
}

// gate/up MXFP8 GEMM whose SiLU(gate)*up epilogue writes the down projection's MXFP8 operand.
int64_t gemm_mxf8_silu_q(torch::Tensor q_out, torch::Tensor sf_out, torch::Tensor xq, torch::Tensor sfa,
                         torch::Tensor wq, torch::Tensor sfb, c10::optional<torch::Tensor> bias, int64_t gate_act) {
  const at::cuda::CUDAGuard rz_guard(q_out.device());
  CHECK_CUDA(xq);
  const int M = xq.size(0), K = xq.size(1), N = wq.size(0);
  TORCH_CHECK(K % 128 == 0 && N % 256 == 0 && wq.size(1) == K, "mxf8 silu_q: K % 128, N % 256");
  TORCH_CHECK(q_out.is_contiguous() && q_out.size(0) == M && q_out.size(1) == N / 2 && q_out.element_size() == 1,
              "q_out: e4m3 [M, N/2]");
  TORCH_CHECK(sf_out.numel() >= static_cast<int64_t>((M + 127) / 128) * (N / 256) * 512, "sf_out too small");
  rz::GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.k_splits = 1;
  p.ldd = q_out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.epi = rz::kEpiSiluMulMx;
  p.gate_act = static_cast<int>(gate_act);
  p.status = status_ptr();
  p.sfa = reinterpret_cast<const uint8_t*>(sfa.data_ptr());
  p.sfb = reinterpret_cast<const uint8_t*>(sfb.data_ptr());
  p.q_out = reinterpret_cast<uint8_t*>(q_out.data_ptr());
  p.sf_out = reinterpret_cast<uint8_t*>(sf_out.data_ptr());
  check_rc(rz::gemm_mxf8_launch(p, xq.data_ptr(), xq.stride(0), wq.data_ptr(), wq.stride(0), 256, cur_stream()),
           "gemm_mxf8_silu_q");
  return 1;
}

std::vector<int64_t> gemm_plan_mxf8(int64_t M, int64_t N, int64_t K, int64_t epi) {
  auto pl = rz::plan_gemm_mxf8(M, N, K, epi);
  return {pl.bn, pl.k_splits};
}

// ---------------------------------------------------------------- MoE
// Grouped GEMM over 128-aligned expert segments: x [rows, K], w [G, N, K] -> out [rows, N or N/2].
int64_t gemm_grouped(torch::Tensor out, torch::Tensor x, torch::Tensor w, torch::Tensor grp_off,
                     torch::Tensor grp_end, int64_t epi, int64_t bn) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w);
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous() && out.is_contiguous(), "grouped gemm: contiguous tensors");
  TORCH_CHECK(w.dim() == 3 && w.size(2) == x.size(1), "grouped gemm: w [G, N, K]");
  const int G = w.size(0), N = w.size(1), K = x.size(1);
  TORCH_CHECK(grp_off.numel() == G + 1 && grp_end.numel() == G && grp_off.scalar_type() == at::kInt,
              "grouped gemm: int32 grp_off [G+1], grp_end [G]");
  TORCH_CHECK(G <= rz::kMaxGemmGroups && K % 64 == 0 && N % 64 == 0, "grouped gemm: G <= 64, K/N multiples of 64");
  if ((epi & 0xff) == rz::kEpiSiluMul) TORCH_CHECK(N % 128 == 0 && out.size(1) == N / 2, "silu epilogue: N % 128, out N/2");
  if (bn <= 0) bn = (static_cast<int64_t>((x.size(0) + 127) / 128) * (N / 256) >= 2 * rz::num_sms()) ? 256 : 128;
  rz::GemmParams p{};
  p.N = N; p.K = K;
  p.k_splits = 1;
  p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldd = out.stride(0);
  p.epi = static_cast<int>(epi & 0xff);
  p.gate_act = static_cast<int>((epi >> 8) & 1);   // kGateGelu: GELU(tanh) gate
  p.status = status_ptr();
  p.grp_off = grp_off.data_ptr<int>();
  p.grp_end = grp_end.data_ptr<int>();
  p.num_groups = G;
  check_rc(rz::gemm_grouped_launch(p, x.data_ptr(), K, x.size(0), w.data_ptr(), K, bn, false, cur_stream()),
           "gemm_grouped");
  return 1;
}

// Local experts of an MoE block: route -> permute -> grouped gate/up (SiLU) -> grouped down.
// w13 holds every local expert's gate/up rows interleaved in 64-row blocks.  Returns (y, pos_of,
// topk_w): expert outputs in expert-sorted rows and, per (token, slot), its row in y (-1 when the
// slot's expert lives on another rank) and gate weight.
struct MoeExpertOut {
  torch::Tensor y, pos, tw;
};
MoeExpertOut moe_experts(torch::Tensor h, torch::Tensor wr, torch::Tensor w13, torch::Tensor w2, int64_t topk,
                         int64_t e_lo, bool renormalize) {
  const at::cuda::CUDAGuard rz_guard(h.device());
  CHECK_CUDA(h); CHECK_BF16(h); CHECK_BF16(wr); CHECK_BF16(w13); CHECK_BF16(w2); CHECK_LAST(h);
  const int M = h.size(0), H = h.size(1), E = wr.size(0), ne = w13.size(0), I = w13.size(1) / 2;
  TORCH_CHECK(wr.size(1) == H && w13.size(2) == H && w2.size(0) == ne && w2.size(1) == H && w2.size(2) == I,
              "moe: weight shapes");
  TORCH_CHECK(topk >= 1 && topk <= 8 && topk <= E && E <= 32 && e_lo >= 0 && e_lo + ne <= E, "moe: expert ranges");
  auto i32 = h.options().dtype(torch::kInt32);
  auto cnt = torch::zeros({2 * ne}, i32);  // counts | fill
  auto tw = torch::empty({M, topk}, h.options().dtype(torch::kFloat32));
  auto tid = torch::empty({M, topk}, i32);
  rz::MoeRouteParams rp{};
  rp.h = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()); rp.ldh = h.stride(0);
  rp.wr = reinterpret_cast<const __nv_bfloat16*>(wr.data_ptr());
  rp.M = M; rp.H = H; rp.E = E; rp.topk = topk; rp.e_lo = e_lo; rp.ne = ne; rp.renormalize = renormalize;
  rp.topk_w = tw.data_ptr<float>(); rp.topk_id = tid.data_ptr<int>(); rp.counts = cnt.data_ptr<int>();
  check_rc(rz::moe_route_launch(rp, cur_stream()), "moe_route");
  const int64_t rows = static_cast<int64_t>(M) * topk + 128 * ne;
  auto x_perm = torch::empty({rows, H}, h.options());
  auto grp = torch::empty({2 * ne + 1}, i32);
  auto pos = torch::empty({M * topk}, i32);
  rz::MoePermuteParams pp{};
  pp.h = rp.h; pp.ldh = rp.ldh; pp.topk_id = rp.topk_id; pp.counts = rp.counts;
  pp.M = M; pp.H = H; pp.topk = topk; pp.e_lo = e_lo; pp.ne = ne;
  pp.fill = rp.counts + ne; pp.grp_off = grp.data_ptr<int>(); pp.grp_end = pp.grp_off + ne + 1;
  pp.pos_of = pos.data_ptr<int>(); pp.x_perm = reinterpret_cast<__nv_bfloat16*>(x_perm.data_ptr());
  check_rc(rz::moe_permute_launch(pp, cur_stream()), "moe_permute");
  auto go = grp.narrow(0, 0, ne + 1), ge = grp.narrow(0, ne + 1, ne);
  auto act = torch::empty({rows, I}, h.options());
  gemm_grouped(act, x_perm, w13, go, ge, rz::kEpiSiluMul, 0);
  auto y = torch::empty({rows, H}, h.options());
  gemm_grouped(y, act, w2, go, ge, rz::kEpiNone, 0);
  return {y, pos, tw};
}

// Whole MoE block for the local experts with the weighted combine on this rank.
// Returns the number of kernels launched.
int64_t moe_forward(torch::Tensor out, torch::Tensor h, torch::Tensor wr, torch::Tensor w13, torch::Tensor w2,
                    int64_t topk, int64_t e_lo, bool renormalize, c10::optional<torch::Tensor> residual) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  const int M = h.size(0), H = h.size(1);
  TORCH_CHECK(out.is_contiguous() && out.size(0) == M && out.size(1) == H, "moe: out [M, H]");
  auto e = moe_experts(h, wr, w13, w2, topk, e_lo, renormalize);
  rz::MoeCombineParams cp{};
  cp.y = reinterpret_cast<const __nv_bfloat16*>(e.y.data_ptr()); cp.ldy = H;
  cp.pos_of = e.pos.data_ptr<int>(); cp.topk_w = e.tw.data_ptr<float>();
  cp.residual = residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  cp.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  cp.M = M; cp.H = H; cp.topk = topk;
  check_rc(rz::moe_combine_launch(cp, cur_stream()), "moe_combine");
  return 6;   // zero-fill, route, permute, 2 grouped GEMMs, combine
}

// Race testing of the flag protocols: random pauses (below this many ns) before the peer
// stores and flag releases of the communication kernels; 0 (default) disables them.
static uint32_t g_comm_jitter_ns = 0;
void set_comm_jitter_ns(int64_t ns) { g_comm_jitter_ns = static_cast<uint32_t>(ns < 0 ? 0 : ns); }

// Expert-parallel MoE block: local experts, then every local (token, slot) output row is sent to
// the token's owner rank (slot buffers + flags over NVLink) for rs_norm_ag in MoE mode.
int64_t moe_forward_peer(torch::Tensor h, torch::Tensor wr, torch::Tensor w13, torch::Tensor w2, int64_t topk,
                         int64_t e_lo, bool renormalize, std::vector<int64_t> slots, std::vector<int64_t> flags,
                         int64_t rs_rows, torch::Tensor epoch, int64_t call_idx) {
  const at::cuda::CUDAGuard rz_guard(h.device());
  const int M = h.size(0), H = h.size(1);
  const int world = static_cast<int>(slots.size());
  TORCH_CHECK(world >= 1 && world <= rz::kMaxTpRanks && flags.size() == slots.size() && topk <= world &&
                  static_cast<int64_t>(rs_rows) * world >= M,
              "moe_forward_peer: ranks / slots");
  auto e = moe_experts(h, wr, w13, w2, topk, e_lo, renormalize);
  rz::MoeCombinePeerParams cp{};
  cp.y = reinterpret_cast<const __nv_bfloat16*>(e.y.data_ptr());
  cp.pos_of = e.pos.data_ptr<int>(); cp.topk_w = e.tw.data_ptr<float>();
  for (int i = 0; i < world; ++i) {
    cp.slot[i] = reinterpret_cast<__nv_bfloat16*>(slots[i]);
    cp.flag[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  cp.M = M; cp.H = H; cp.topk = topk; cp.rs_rows = rs_rows;
  cp.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  cp.call_idx = static_cast<uint32_t>(call_idx);
  cp.jitter_ns = g_comm_jitter_ns;
  check_rc(rz::moe_combine_peer_launch(cp, cur_stream()), "moe_combine_peer");
  return 6;
}

void ag_wait(torch::Tensor ag_flag, int64_t M, torch::Tensor epoch, int64_t call_idx) {
  const at::cuda::CUDAGuard rz_guard(ag_flag.device());
  check_rc(rz::ag_wait_launch(reinterpret_cast<const uint32_t*>(ag_flag.data_ptr()), M,
                              reinterpret_cast<const uint32_t*>(epoch.data_ptr()), static_cast<uint32_t>(call_idx),
                              status_ptr(), cur_stream()),
           "ag_wait");
}

// Routing only (tests): fills topk weights / ids and the local expert counts.
void moe_route(torch::Tensor tw, torch::Tensor tid, torch::Tensor counts, torch::Tensor h, torch::Tensor wr,
               int64_t topk, int64_t e_lo, int64_t ne, bool renormalize) {
  const at::cuda::CUDAGuard rz_guard(tw.device());
  CHECK_CUDA(h); CHECK_BF16(h); CHECK_BF16(wr);
  rz::MoeRouteParams rp{};
  rp.h = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()); rp.ldh = h.stride(0);
  rp.wr = reinterpret_cast<const __nv_bfloat16*>(wr.data_ptr());
  rp.M = h.size(0); rp.H = h.size(1); rp.E = wr.size(0); rp.topk = topk; rp.e_lo = e_lo; rp.ne = ne;
  rp.renormalize = renormalize;
  rp.topk_w = tw.data_ptr<float>(); rp.topk_id = tid.data_ptr<int>(); rp.counts = counts.data_ptr<int>();
  check_rc(rz::moe_route_launch(rp, cur_stream()), "moe_route");
}

// ---------------------------------------------------------------- fused tensor-parallel boundary

// Row-parallel GEMM whose epilogue reduce-scatters into the owners' slot buffers.  Returns n_tiles.
int64_t gemm_peer_rs(torch::Tensor x, torch::Tensor w, std::vector<int64_t> slots, std::vector<int64_t> flags,
                     int64_t rank, int64_t rs_rows, torch::Tensor epoch, int64_t call_idx, int64_t bn) {
  const at::cuda::CUDAGuard rz_guard(x.device());
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w); CHECK_LAST(x); CHECK_LAST(w);
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  const int world = static_cast<int>(slots.size());
  TORCH_CHECK(world >= 1 && world <= rz::kMaxTpRanks && flags.size() == slots.size(), "gemm_peer_rs: 1..8 ranks");
  TORCH_CHECK(w.size(1) == K && K % 8 == 0 && N % 8 == 0 && rs_rows % rz::kAgRowBlock == 0 &&
                  static_cast<int64_t>(rs_rows) * world >= M,
              "gemm_peer_rs: shapes");
  if (bn <= 0) bn = rz::plan_gemm(M, N, K, 0, /*max_splits=*/1).bn;   // the epilogue stores final rows
  rz::GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.k_splits = 1;
  p.epi = rz::kEpiPeerRS;
  p.status = status_ptr();
  for (int i = 0; i < world; ++i) {
    p.rs_slot[i] = reinterpret_cast<__nv_bfloat16*>(slots[i]);
    p.rs_flag[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  p.rs_rows = rs_rows;
  p.tp_rank = rank; p.tp_world = world;
  p.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  p.call_idx = static_cast<uint32_t>(call_idx);
  p.jitter_ns = g_comm_jitter_ns;
  check_rc(rz::gemm_bf16_launch(p, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), bn, cur_stream()),
           "gemm_peer_rs");
  return (N + bn - 1) / bn;
}

// GEMM whose A rows are all-gathered by peers: waits on the local all-gather flags per A tile.
int64_t gemm_ag(torch::Tensor out, torch::Tensor g, torch::Tensor w, c10::optional<torch::Tensor> bias, int64_t epi,
                torch::Tensor ag_flag, torch::Tensor epoch, int64_t call_idx) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(g); CHECK_BF16(g); CHECK_BF16(w); CHECK_LAST(g); CHECK_LAST(w);
  const int M = g.size(0), K = g.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && K % 8 == 0 && N % 8 == 0, "gemm_ag: shapes");
  if ((epi & 0xff) == rz::kEpiSiluMul) TORCH_CHECK(N % 128 == 0 && out.size(1) == N / 2, "silu epilogue: N % 128, out N/2");
  auto pl = rz::plan_gemm(M, N, K, static_cast<int>(epi & 0xff));
  rz::GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.k_splits = pl.k_splits;
  p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldd = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.epi = static_cast<int>(epi & 0xff);
  p.gate_act = static_cast<int>((epi >> 8) & 1);   // kGateGelu: GELU(tanh) gate
  p.status = status_ptr();
  p.ag_flag = reinterpret_cast<const uint32_t*>(ag_flag.data_ptr());
  p.ag_rows = M;
  p.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  p.call_idx = static_cast<uint32_t>(call_idx);
  torch::Tensor ws;
  if (pl.k_splits > 1) {
    ws = torch::empty({pl.k_splits, M, N}, g.options().dtype(torch::kFloat32));
    p.partial = ws.data_ptr<float>();
  }
  check_rc(rz::gemm_bf16_launch(p, g.data_ptr(), g.stride(0), w.data_ptr(), w.stride(0), pl.bn, cur_stream()),
           "gemm_ag");
  return pl.k_splits > 1 ? 2 : 1;
}

// MXFP8 row-parallel GEMM whose epilogue reduce-scatters bf16 rows into the owners' slots.
// Returns n_tiles.
int64_t gemm_peer_rs_mx(torch::Tensor xq, torch::Tensor sfa, torch::Tensor wq, torch::Tensor wsf,
                        std::vector<int64_t> slots, std::vector<int64_t> flags, int64_t rank, int64_t rs_rows,
                        torch::Tensor epoch, int64_t call_idx) {
  const at::cuda::CUDAGuard rz_guard(xq.device());
  CHECK_CUDA(xq);
  const int M = xq.size(0), K = xq.size(1), N = wq.size(0);
  const int world = static_cast<int>(slots.size());
  TORCH_CHECK(world >= 1 && world <= rz::kMaxTpRanks && flags.size() == slots.size(), "gemm_peer_rs_mx: 1..8 ranks");
  TORCH_CHECK(K % 128 == 0 && N % 128 == 0 && wq.size(1) == K && xq.is_contiguous() && wq.is_contiguous() &&
                  xq.element_size() == 1 && wq.element_size() == 1,
              "gemm_peer_rs_mx: contiguous e4m3 [M,K] x [N,K], K and N multiples of 128");
  TORCH_CHECK(rs_rows % rz::kAgRowBlock == 0 && static_cast<int64_t>(rs_rows) * world >= M, "gemm_peer_rs_mx: rows");
  const int bn = rz::plan_gemm_mxf8(M, N, K, 0, /*max_splits=*/1).bn;   // the epilogue stores final rows
  rz::GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.k_splits = 1;
  p.epi = rz::kEpiPeerRS;
  p.status = status_ptr();
  p.sfa = reinterpret_cast<const uint8_t*>(sfa.data_ptr());
  p.sfb = reinterpret_cast<const uint8_t*>(wsf.data_ptr());
  for (int i = 0; i < world; ++i) {
    p.rs_slot[i] = reinterpret_cast<__nv_bfloat16*>(slots[i]);
    p.rs_flag[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  p.rs_rows = rs_rows;
  p.tp_rank = rank; p.tp_world = world;
  p.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  p.call_idx = static_cast<uint32_t>(call_idx);
  p.jitter_ns = g_comm_jitter_ns;
  check_rc(rz::gemm_mxf8_launch(p, xq.data_ptr(), xq.stride(0), wq.data_ptr(), wq.stride(0), bn, cur_stream()),
           "gemm_peer_rs_mx");
  return (N + bn - 1) / bn;
}

// MXFP8 GEMM on all-gathered operand rows (e4m3 + scale chunks written by the owners): the
// TMA producer waits on the all-gather flags per A tile.  silu_q: gate/up with the SiLU
// epilogue emitting the next MXFP8 operand into (out, sf_out); else bf16 rows into out.
int64_t gemm_mxf8_ag(torch::Tensor out, c10::optional<torch::Tensor> sf_out, torch::Tensor gq, torch::Tensor gsf,
                     torch::Tensor wq, torch::Tensor wsf, c10::optional<torch::Tensor> bias, torch::Tensor ag_flag,
                     torch::Tensor epoch, int64_t call_idx) {
  const at::cuda::CUDAGuard rz_guard(out.device());
  CHECK_CUDA(gq);
  const int M = gq.size(0), K = gq.size(1), N = wq.size(0);
  const bool silu_q = sf_out.has_value();
  TORCH_CHECK(K % 128 == 0 && N % (silu_q ? 256 : 128) == 0 && wq.size(1) == K && wq.is_contiguous() &&
                  gq.element_size() == 1 && wq.element_size() == 1,
              "gemm_mxf8_ag: e4m3 [M,K] x [N,K], K % 128, N % 128 (256 with silu_q)");
  rz::GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  int bn = 256;
  if (silu_q) {
    TORCH_CHECK(out.size(0) == M && out.size(1) == N / 2 && out.element_size() == 1, "gemm_mxf8_ag: q_out [M, N/2]");
    p.k_splits = 1;
    p.epi = rz::kEpiSiluMulMx;
    p.ldd = out.stride(0);
    p.q_out = reinterpret_cast<uint8_t*>(out.data_ptr());
    p.sf_out = reinterpret_cast<uint8_t*>(sf_out->data_ptr());
  } else {
    auto pl = rz::plan_gemm_mxf8(M, N, K, 0);
    bn = pl.bn;
    p.k_splits = pl.k_splits;
    p.epi = rz::kEpiNone;
    p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    p.ldd = out.stride(0);
  }
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.status = status_ptr();
  p.sfa = reinterpret_cast<const uint8_t*>(gsf.data_ptr());
  p.sfb = reinterpret_cast<const uint8_t*>(wsf.data_ptr());
  p.ag_flag = reinterpret_cast<const uint32_t*>(ag_flag.data_ptr());
  p.ag_rows = M;
  p.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  p.call_idx = static_cast<uint32_t>(call_idx);
  torch::Tensor ws;
  if (p.k_splits > 1) {
    ws = torch::empty({p.k_splits, M, N}, wq.options().dtype(torch::kFloat32));
    p.partial = ws.data_ptr<float>();
  }
  check_rc(rz::gemm_mxf8_launch(p, gq.data_ptr(), gq.stride(0), wq.data_ptr(), wq.stride(0), bn, cur_stream()),
           "gemm_mxf8_ag");
  return p.k_splits > 1 ? 2 : 1;
}

void rs_norm_ag(torch::Tensor slots, torch::Tensor rs_flag, int64_t n_tiles, c10::optional<torch::Tensor> resid_in,
                torch::Tensor residual, torch::Tensor w, double eps, double offset, std::vector<int64_t> gathers,
                std::vector<int64_t> ag_flags, int64_t rank, int64_t M, int64_t rs_rows, torch::Tensor epoch,
                int64_t call_idx, int64_t moe_topk, c10::optional<torch::Tensor> moe_flag,
                std::vector<int64_t> gathers_q, std::vector<int64_t> gathers_sf) {
  const at::cuda::CUDAGuard rz_guard(slots.device());
  CHECK_BF16(residual); CHECK_BF16(w);
  const int world = static_cast<int>(gathers.size());
  TORCH_CHECK(world >= 1 && world <= rz::kMaxTpRanks && ag_flags.size() == gathers.size(), "rs_norm_ag: ranks");
  rz::RsNormAgParams p{};
  p.slots = reinterpret_cast<const __nv_bfloat16*>(slots.data_ptr());
  p.rs_flag = reinterpret_cast<const uint32_t*>(rs_flag.data_ptr());
  p.n_tiles = n_tiles;
  p.reduce = resid_in.has_value() ? 0 : 1;
  p.resid_in = resid_in.has_value() ? reinterpret_cast<const __nv_bfloat16*>(resid_in->data_ptr()) : nullptr;
  p.residual = reinterpret_cast<__nv_bfloat16*>(residual.data_ptr());
  p.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  p.eps = eps; p.offset = offset;
  for (int i = 0; i < world; ++i) {
    p.gather[i] = reinterpret_cast<__nv_bfloat16*>(gathers[i]);
    p.ag_flag[i] = reinterpret_cast<uint32_t*>(ag_flags[i]);
  }
  p.rank = rank; p.world = world; p.M = M; p.rs_rows = rs_rows; p.H = w.size(0);
  p.epoch_ptr = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  p.call_idx = static_cast<uint32_t>(call_idx);
  p.status = status_ptr();
  p.moe_topk = static_cast<int>(moe_topk);
  if (moe_topk > 0) {
    TORCH_CHECK(moe_flag.has_value(), "rs_norm_ag: MoE mode needs the moe flags");
    p.moe_flag = reinterpret_cast<const uint32_t*>(moe_flag->data_ptr());
  }
  p.jitter_ns = g_comm_jitter_ns;
  p.mx = gathers_q.empty() ? 0 : 1;
  if (p.mx) {
    TORCH_CHECK(gathers_q.size() == gathers.size() && gathers_sf.size() == gathers.size(),
                "rs_norm_ag: one MXFP8 gather buffer pair per rank");
    for (int i = 0; i < world; ++i) {
      p.gather_q[i] = reinterpret_cast<uint8_t*>(gathers_q[i]);
      p.gather_sf[i] = reinterpret_cast<uint8_t*>(gathers_sf[i]);
    }
  }
  check_rc(rz::rs_norm_ag_launch(p, cur_stream()), "rs_norm_ag");
}

void tp_epoch_bump(torch::Tensor epoch) {
  const at::cuda::CUDAGuard rz_guard(epoch.device());
  check_rc(rz::tp_epoch_bump_launch(reinterpret_cast<uint32_t*>(epoch.data_ptr()), cur_stream()), "tp_epoch_bump");
}

// ---------------------------------------------------------------- sampling
// ----------------------------------------------------------------------------- cluster sampler
// Slot tables, in order: f32 [S,8], i32 [S,8], n_gen [S], seed [S], cnt [P, ceil(V/2)] (may be
// empty), seen [P, ceil(V/32)] (may be empty), bias_tok [S, kSampMaxBias], bias_val, stop_ids.
static rz::SampleSlotTables slot_tables(const std::vector<torch::Tensor>& t) {
  TORCH_CHECK(t.size() == 9, "nine slot tables expected");
  rz::SampleSlotTables st{};
  st.f32 = t[0].data_ptr<float>();
  st.i32 = t[1].data_ptr<int32_t>();
  st.n_gen = t[2].data_ptr<int32_t>();
  st.seed = t[3].data_ptr<int64_t>();
  st.cnt = t[4].numel() ? reinterpret_cast<uint32_t*>(t[4].data_ptr<int32_t>()) : nullptr;
  st.seen = t[5].numel() ? reinterpret_cast<uint32_t*>(t[5].data_ptr<int32_t>()) : nullptr;
  st.bias_tok = t[6].data_ptr<int32_t>();
  st.bias_val = t[7].data_ptr<float>();
  st.stop_ids = t[8].data_ptr<int32_t>();
  return st;
}

static rz::SampleClusterArgs cluster_args(torch::Tensor tok, torch::Tensor lp, torch::Tensor logits) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits [R, V] with unit column stride");
  TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16, "fp32 or bf16 logits");
  rz::SampleClusterArgs a{};
  a.logits = logits.data_ptr();
  a.ld = logits.stride(0);
  a.R = static_cast<int>(logits.size(0));
  a.V = static_cast<int>(logits.size(1));
  a.tok = tok.data_ptr<int64_t>();
  a.lp = lp.data_ptr<float>();
  return a;
}

// Per-row parameters (every row greedy when temp <= 0).
void sample_rows(torch::Tensor tok, torch::Tensor lp, torch::Tensor logits, torch::Tensor temp, torch::Tensor topk,
                 torch::Tensor topp, torch::Tensor minp, torch::Tensor seeds, torch::Tensor offsets) {
  const at::cuda::CUDAGuard rz_guard(tok.device());
  rz::SampleClusterArgs a = cluster_args(tok, lp, logits);
  a.temp = temp.data_ptr<float>();
  a.topk = topk.data_ptr<int32_t>();
  a.topp = topp.data_ptr<float>();
  a.minp = minp.data_ptr<float>();
  a.seeds = seeds.data_ptr<int64_t>();
  a.offsets = offsets.data_ptr<int64_t>();
  check_rc(rz::sample_cluster_launch(a, logits.scalar_type() == at::kBFloat16, false, cur_stream()), "sample_rows");
}

// Slot mode: row_info[r] = slot | (sample index << 16); penalties, bias and min_tokens from the
// tables; the kernel advances each slot's generated count and penalty counts.
void sample_slots(torch::Tensor tok, torch::Tensor lp, torch::Tensor logits, torch::Tensor row_info,
                  std::vector<torch::Tensor> tables) {
  const at::cuda::CUDAGuard rz_guard(tok.device());
  rz::SampleClusterArgs a = cluster_args(tok, lp, logits);
  TORCH_CHECK(row_info.scalar_type() == at::kInt && row_info.numel() >= a.R, "row_info int32 [R]");
  a.row_info = row_info.data_ptr<int32_t>();
  a.st = slot_tables(tables);
  check_rc(rz::sample_cluster_launch(a, logits.scalar_type() == at::kBFloat16, true, cur_stream()), "sample_slots");
}

void sample_slot_init(std::vector<torch::Tensor> tables, int64_t n, int64_t V, torch::Tensor slot, torch::Tensor f32,
                      torch::Tensor i32, torch::Tensor n_gen, torch::Tensor seed, torch::Tensor bias_tok,
                      torch::Tensor bias_val, torch::Tensor stop_ids, torch::Tensor tok_off, torch::Tensor toks) {
  const at::cuda::CUDAGuard rz_guard(slot.device());
  rz::SampleSlotInit u{};
  u.slot = slot.data_ptr<int32_t>();
  u.f32 = f32.data_ptr<float>();
  u.i32 = i32.data_ptr<int32_t>();
  u.n_gen = n_gen.data_ptr<int32_t>();
  u.seed = seed.data_ptr<int64_t>();
  u.bias_tok = bias_tok.data_ptr<int32_t>();
  u.bias_val = bias_val.data_ptr<float>();
  u.stop_ids = stop_ids.data_ptr<int32_t>();
  u.tok_off = tok_off.data_ptr<int32_t>();
  u.toks = toks.data_ptr<int32_t>();
  check_rc(rz::sample_slot_init_launch(u, static_cast<int>(n), slot_tables(tables), static_cast<int>(V), cur_stream()),
           "sample_slot_init");
}

void spec_verify(torch::Tensor out_tokens, torch::Tensor n_acc, torch::Tensor target_logits,
                 c10::optional<torch::Tensor> draft_logits, torch::Tensor draft_tokens, torch::Tensor temp,
                 torch::Tensor seeds, torch::Tensor offsets) {
  const at::cuda::CUDAGuard rz_guard(out_tokens.device());
  const int B = draft_tokens.size(0), k = draft_tokens.size(1);
  const int V = target_logits.size(1);
  TORCH_CHECK(target_logits.size(0) == B * (k + 1), "target logits must have B*(k+1) rows");
  const float* dl = nullptr;
  if (draft_logits.has_value()) {
    TORCH_CHECK(draft_logits->stride(0) == target_logits.stride(0), "draft/target logits must share a row stride");
    dl = draft_logits->data_ptr<float>();
  }
  check_rc(rz::spec_verify_launch(target_logits.data_ptr<float>(), dl, draft_tokens.data_ptr<int64_t>(), B, k, V,
                                  target_logits.stride(0), temp.data_ptr<float>(), seeds.data_ptr<int64_t>(),
                                  offsets.data_ptr<int64_t>(), out_tokens.data_ptr<int64_t>(),
                                  n_acc.data_ptr<int32_t>(), cur_stream()),
           "spec_verify");
}

void copy_blocks(torch::Tensor cache, torch::Tensor pairs) {
  const at::cuda::CUDAGuard rz_guard(cache.device());
  TORCH_CHECK(pairs.scalar_type() == at::kInt && pairs.is_cuda(), "int32 CUDA pairs");
  const int64_t block_bytes = cache.stride(0) * cache.element_size();
  check_rc(rz::copy_blocks_launch(cache.data_ptr(), pairs.data_ptr<int32_t>(), pairs.size(0), block_bytes,
                                  cur_stream()),
           "copy_blocks");
}

torch::Tensor read_status() {
  int dev;
  cudaGetDevice(&dev);
  return status_tensor(dev);
}

}  // namespace

void bind_comm(pybind11::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "rusteeze_b200 sm_100a kernels";
  m.def("rms_norm", &rms_norm);
  m.def("fused_add_rms_norm", &fused_add_rms_norm);
  m.def("rope_and_cache", &rope_and_cache, py::arg("qkv"), py::arg("positions"), py::arg("cos_sin"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("slots"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"),
        py::arg("k_scale") = 1.0, py::arg("v_scale") = 1.0);
  m.def("act_mul", &act_mul);
  m.def("embedding", &embedding);
  m.def("layer_norm", &layer_norm);
  m.def("decode_attention", &decode_attention, py::arg("out"), py::arg("q"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("seq_lens"), py::arg("block_tables"), py::arg("workspace"),
        py::arg("num_seqs"), py::arg("scale"), py::arg("window"), py::arg("softcap"), py::arg("num_splits"),
        py::arg("alibi") = py::none(), py::arg("k_scale") = 1.0, py::arg("v_scale") = 1.0);
  m.def("kv_dequant_gather", &kv_dequant_gather);
  m.def("prefill_attention", &prefill_attention, py::arg("out"), py::arg("q"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("qsl"), py::arg("seq_lens"), py::arg("block_tables"), py::arg("seq_offset"),
        py::arg("num_seqs"), py::arg("max_q_len"), py::arg("scale"), py::arg("window"), py::arg("softcap"),
        py::arg("alibi") = py::none());
  m.def("prefill_attention_impl", &prefill_attention_impl, py::arg("out"), py::arg("q"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("qsl"), py::arg("seq_lens"), py::arg("block_tables"), py::arg("seq_offset"),
        py::arg("num_seqs"), py::arg("max_q_len"), py::arg("scale"), py::arg("window"), py::arg("softcap"),
        py::arg("impl"), py::arg("alibi") = py::none());
  m.def("gemm_plan", &gemm_plan);
  m.def("gemm_bf16", &gemm_bf16);
  m.def("gemm_bf16_ex", &gemm_bf16_ex);
  m.def("quant_fp8_act", &quant_fp8_act);
  m.def("gemm_fp8_block", &gemm_fp8_block);
  m.def("quant_mxf8_act", &quant_mxf8_act);
  m.def("rms_norm_mxf8", &rms_norm_mxf8);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("gemm_peer_rs", &gemm_peer_rs);
  m.def("gemm_ag", &gemm_ag);
  namespace py = pybind11;
  m.def("rs_norm_ag", &rs_norm_ag, py::arg("slots"), py::arg("rs_flag"), py::arg("n_tiles"), py::arg("resid_in"),
        py::arg("residual"), py::arg("w"), py::arg("eps"), py::arg("offset"), py::arg("gathers"),
        py::arg("ag_flags"), py::arg("rank"), py::arg("M"), py::arg("rs_rows"), py::arg("epoch"),
        py::arg("call_idx"), py::arg("moe_topk"), py::arg("moe_flag"),
        py::arg("gathers_q") = std::vector<int64_t>{}, py::arg("gathers_sf") = std::vector<int64_t>{});
  m.def("gemm_peer_rs_mx", &gemm_peer_rs_mx);
  m.def("set_comm_jitter_ns", &set_comm_jitter_ns);
  m.def("gemm_mxf8_ag", &gemm_mxf8_ag);
  m.def("moe_forward_peer", &moe_forward_peer);
  m.def("ag_wait", &ag_wait);
  m.def("tp_epoch_bump", &tp_epoch_bump);
  m.def("moe_forward", &moe_forward);
  m.def("moe_route", &moe_route);
  m.def("gemm_mxf8", &gemm_mxf8);
  m.def("gemm_plan_mxf8", &gemm_plan_mxf8);
  m.def("gemm_mxf8_silu_q", &gemm_mxf8_silu_q, py::arg("q_out"), py::arg("sf_out"), py::arg("xq"), py::arg("sfa"),
        py::arg("wq"), py::arg("sfb"), py::arg("bias"), py::arg("gate_act") = 0);
  m.def("spec_verify", &spec_verify);
  m.def("sample_rows", &sample_rows);
  m.def("sample_slots", &sample_slots);
  m.def("sample_slot_init", &sample_slot_init);
  m.attr("SAMPLE_MAX_BIAS") = rz::kSampMaxBias;
  m.attr("SAMPLE_MAX_STOP") = rz::kSampMaxStop;
  m.def("copy_blocks", &copy_blocks);
  m.def("status", &read_status);
  bind_comm(m);
}
