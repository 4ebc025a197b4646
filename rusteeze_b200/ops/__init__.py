"""Device ops used by the models and engine.

Every op has exactly two implementations:
  * CUDA tensors  -> the hand-written sm_100a kernels in `rusteeze_b200._C`
                     (built from csrc/kernels/*.cu).  If the extension is not
                     built, calling an op on a CUDA tensor raises; there is no
                     silent eager fallback on the GPU.
  * CPU tensors   -> the fp32 PyTorch oracle in `ops.reference`, which is also
                     what the numerics tests compare the kernels against.
"""
from __future__ import annotations

import importlib
from typing import Optional

import torch

from rusteeze_b200.ops import reference as ref
from rusteeze_b200.ops.reference import BLOCK_SIZE  # noqa: F401

_C = None
_C_ERR: Optional[BaseException] = None


def cuda_ext():
    """The compiled kernel extension; raises loudly if it is missing."""
    global _C, _C_ERR
    if _C is None:
        try:
            _C = importlib.import_module("rusteeze_b200._C")
        except BaseException as e:  # noqa: BLE001
            _C_ERR = e
            raise RuntimeError(
                "rusteeze_b200._C (sm_100a kernels) is not built or failed to load; run "
                "`python setup.py build_ext --inplace` (or __graft_entry__.build()). "
                f"Underlying error: {e!r}") from e
    return _C


def ext_available() -> bool:
    try:
        cuda_ext()
        return True
    except RuntimeError:
        return False


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


# Number of this package's kernels launched so far (graph replays add the
# count recorded at capture time).  Benchmarks report the delta.
_LAUNCHES = [0]


def launch_count() -> int:
    return _LAUNCHES[0]


def add_launches(n: int) -> None:
    _LAUNCHES[0] += n


# ----------------------------------------------------------------------------- norms
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, offset: float = 0.0) -> torch.Tensor:
    if not x.is_cuda:
        return ref.rms_norm(x, w, eps, offset)
    out = torch.empty_like(x)
    cuda_ext().rms_norm(out, x, w, float(eps), float(offset))
    _LAUNCHES[0] += 1
    return out


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                       offset: float = 0.0):
    """residual += x (in place); returns (rms_norm(residual), residual)."""
    if not x.is_cuda:
        out, r = ref.fused_add_rms_norm(x, residual, w, eps, offset)
        residual.copy_(r)
        return out, residual
    out = torch.empty_like(x)
    cuda_ext().fused_add_rms_norm(out, x, residual, w, float(eps), float(offset))
    _LAUNCHES[0] += 1
    return out, residual


# ----------------------------------------------------------------------------- rope + kv write
def rope_and_cache(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, slot_mapping: torch.Tensor,
                   num_q_heads: int, num_kv_heads: int, head_dim: int, k_scale: float = 1.0,
                   v_scale: float = 1.0) -> torch.Tensor:
    """Applies neox RoPE to the q and k parts of the fused qkv [T, (Hq+2Hkv)*D]
    output (q in place), writes rotated k and v into the paged caches at
    slot_mapping, and returns q as a [T, Hq, D] view.  fp8 caches (float8_e4m3fn /
    float8_e5m2) store k / k_scale and v / v_scale, saturated."""
    T = qkv.shape[0]
    qs, kvs = num_q_heads * head_dim, num_kv_heads * head_dim
    if not qkv.is_cuda:
        q = qkv[:, :qs].view(T, num_q_heads, head_dim)
        k = qkv[:, qs:qs + kvs].reshape(T, num_kv_heads, head_dim).clone()
        v = qkv[:, qs + kvs:].reshape(T, num_kv_heads, head_dim)
        qq = q.clone()
        ref.rope(qq, k, positions, cos_sin)
        q.copy_(qq)
        ref.reshape_and_cache(k, v, k_cache, v_cache, slot_mapping, k_scale, v_scale)
        return q
    cuda_ext().rope_and_cache(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping,
                              num_q_heads, num_kv_heads, head_dim, float(k_scale), float(v_scale))
    _LAUNCHES[0] += 1
    return qkv[:, :qs].view(T, num_q_heads, head_dim)


# ----------------------------------------------------------------------------- activations
def embedding(ids: torch.Tensor, table: torch.Tensor, lo: int = 0, vocab: Optional[int] = None,
              scale: float = 1.0) -> torch.Tensor:
    """Rows of a (vocab-parallel) embedding table: table holds vocabulary rows [lo, lo +
    rows); ids outside that range give zero rows (another rank's share), every row is
    multiplied by `scale` (Gemma's sqrt(hidden))."""
    hi = lo + table.shape[0]
    vocab = hi if vocab is None else vocab
    if not ids.is_cuda:
        local = ids - lo
        ok = (local >= 0) & (local < table.shape[0])
        h = table[local.clamp(0, table.shape[0] - 1)] * ok.unsqueeze(1).to(table.dtype)
        return h * torch.tensor(scale, dtype=table.dtype) if scale != 1.0 else h
    out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    if ids.numel():
        cuda_ext().embedding(out, table, ids.contiguous().view(-1), lo, hi, vocab, float(scale))
        _LAUNCHES[0] += 1
    return out


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], eps: float,
               residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LayerNorm with fp32 statistics (bias optional); with `residual`, residual += x first
    (in place) and the sum is normalised."""
    if not x.is_cuda:
        if residual is not None:
            residual.add_(x)
            x = residual
        return ref.layer_norm(x, w, b, eps).to(x.dtype)
    out = torch.empty_like(x)
    if x.shape[0]:
        cuda_ext().layer_norm(out, x.contiguous(), residual, w, b, float(eps))
        _LAUNCHES[0] += 1
    return out


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return ref.silu_mul(x)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
    cuda_ext().act_mul(out, x, 0)
    _LAUNCHES[0] += 1
    return out


def gelu_tanh_mul(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        return ref.gelu_tanh_mul(x)
    out = torch.empty(x.shape[0], x.shape[1] // 2, dtype=x.dtype, device=x.device)
    cuda_ext().act_mul(out, x, 1)
    _LAUNCHES[0] += 1
    return out


# ----------------------------------------------------------------------------- attention
def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, meta,
                    scale: float, sliding_window: Optional[int] = None,
                    softcap: Optional[float] = None,
                    alibi: Optional[torch.Tensor] = None, k_scale: float = 1.0,
                    v_scale: float = 1.0) -> torch.Tensor:
    """q [T, Hq, D] -> out [T, Hq, D].  `meta` is an AttentionMetadata; `alibi` holds
    one fp32 ALiBi slope per query head (None: no positional bias).  With an fp8 cache the
    decode rows read it directly (f16 tensor-core variant) and the other rows read a bf16
    scratch copy of their sequences' blocks (`kv_dequant_gather`)."""
    if not q.is_cuda:
        return ref.paged_attention(q, k_cache, v_cache, meta.query_start_loc, meta.seq_lens,
                                   meta.block_tables, scale, sliding_window, softcap, alibi,
                                   k_scale, v_scale)
    out = torch.empty_like(q)
    C = cuda_ext()
    nd = meta.num_decode_seqs
    win = int(sliding_window or 0)
    cap = float(softcap or 0.0)
    if nd > 0:
        C.decode_attention(out, q, k_cache, v_cache, meta.seq_lens, meta.block_tables,
                           meta.decode_workspace, nd, float(scale), win, cap,
                           meta.decode_num_splits, alibi, float(k_scale), float(v_scale))
        _LAUNCHES[0] += 2 if meta.decode_num_splits > 1 else 1
    if meta.num_seqs > nd:
        kc, vc, bt = k_cache, v_cache, meta.block_tables
        if ref.is_fp8(k_cache.dtype):
            kc, vc, bt = _gather_fp8_kv(k_cache, v_cache, meta, nd, k_scale, v_scale)
        C.prefill_attention(out, q, kc, vc, meta.query_start_loc, meta.seq_lens,
                            bt, nd, meta.num_seqs - nd, meta.max_query_len,
                            float(scale), win, cap, alibi)
        _LAUNCHES[0] += 1
    return out


def _gather_fp8_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, meta, nd: int, k_scale: float,
                   v_scale: float):
    """bf16 scratch pages [prefill_kv_blocks, Hkv, 16, D] for the non-decode sequences and
    their block table (rows indexed like meta.block_tables)."""
    nblk = max(int(meta.prefill_kv_blocks), 1)
    shape = (nblk,) + tuple(k_cache.shape[1:])
    scr = getattr(meta, "_fp8_scratch", None)      # reused by every layer of the forward
    if scr is None or scr[0].shape != shape:
        scr = (torch.empty(shape, dtype=torch.bfloat16, device=k_cache.device),
               torch.empty(shape, dtype=torch.bfloat16, device=k_cache.device),
               torch.zeros_like(meta.block_tables))
        meta._fp8_scratch = scr
    kc, vc, bt = scr
    cuda_ext().kv_dequant_gather(kc, vc, bt, k_cache, v_cache, meta.block_tables, meta.seq_lens, nd,
                                 meta.num_seqs - nd, float(k_scale), float(v_scale))
    _LAUNCHES[0] += 1
    return kc, vc, bt


# ----------------------------------------------------------------------------- gemm
def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
           residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ w.T (+ bias) (+ residual).  x [M, K] bf16, w [N, K] bf16 (K-major).

    On CUDA this is the tcgen05/TMEM GEMM (TMA-fed, no cluster multicast) with
    bias and residual fused into the epilogue."""
    if not x.is_cuda:
        y = ref.linear(x, w, bias)
        if residual is not None:
            y = (y.float() + residual.float()).to(y.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    M, N = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    if M == 0:
        return out
    _LAUNCHES[0] += cuda_ext().gemm_bf16(out, x, w, bias, residual)
    return out


def interleave_gate_up(w: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[gate(I) | up(I)] rows -> [g0:64 | u0:64 | g64:128 | u64:128 | ...], the
    layout the GEMM's SiLU(gate)*up epilogue consumes tile by tile."""
    two_i, K = w.shape
    I = two_i // 2
    assert I % block == 0
    g, u = w[:I].view(I // block, block, K), w[I:].view(I // block, block, K)
    return torch.stack([g, u], dim=1).reshape(two_i, K).contiguous()


def deinterleave_gate_up(w_il: torch.Tensor, block: int = 64) -> torch.Tensor:
    two_i, K = w_il.shape
    I = two_i // 2
    v = w_il.view(I // block, 2, block, K)
    return torch.cat([v[:, 0].reshape(I, K), v[:, 1].reshape(I, K)], dim=0)


GATE_GELU = 1 << 8     # epilogue flag: GELU(tanh) instead of SiLU as the gate activation


def _gate(act: str) -> int:
    if act in ("silu", "swiglu"):
        return 0
    if act in ("gelu_tanh", "gelu", "gelu_pytorch_tanh", "geglu"):
        return GATE_GELU
    raise ValueError(f"unsupported gate activation {act!r}")


def linear_silu_mul(x: torch.Tensor, w_il: torch.Tensor, act: str = "silu") -> torch.Tensor:
    """act(x @ Wg.T) * (x @ Wu.T) in one GEMM (act: SiLU, or GELU-tanh for GeGLU MLPs);
    w_il from interleave_gate_up."""
    M = x.shape[0]
    out = torch.empty(M, w_il.shape[0] // 2, dtype=x.dtype, device=x.device)
    if M == 0:
        return out
    _LAUNCHES[0] += cuda_ext().gemm_bf16_ex(out, x, w_il, None, None, 1 | _gate(act), 0, 0)
    return out


def _act_mul_interleaved(y: torch.Tensor, act: str) -> torch.Tensor:
    """act(gate) * up on GEMM output whose columns are interleaved [gate 64 | up 64] blocks:
    every 128-column block is one [gate | up] row of the activation kernel."""
    M, N = y.shape
    out = torch.empty(M, N // 2, dtype=y.dtype, device=y.device)
    if M:
        cuda_ext().act_mul(out.view(M * (N // 128), 64), y.view(M * (N // 128), 128), 0 if _gate(act) == 0 else 1)
        _LAUNCHES[0] += 1
    return out


def quant_fp8_act(x: torch.Tensor):
    """bf16 [M, K] -> (e4m3 [M, K], fp32 scales [K/128, M]) with 1x128 groups."""
    M, K = x.shape
    if not x.is_cuda:
        q, s = ref.quant_fp8_act(x)
        return q, s.t().contiguous()
    xq = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    xs = torch.empty(K // 128, M, dtype=torch.float32, device=x.device)
    if M:
        cuda_ext().quant_fp8_act(xq, xs, x)
        _LAUNCHES[0] += 1
    return xq, xs


def quant_mxf8_act(x: torch.Tensor):
    """bf16 [M, K] -> (e4m3 [M, K], uint8 scale chunks [ceil(M/128), K/128, 512])
    with power-of-two 1x128 scales in the block-scaled MMA's TMEM copy layout."""
    M, K = x.shape
    xq = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    sfa = torch.empty((M + 127) // 128, K // 128, 512, dtype=torch.uint8, device=x.device)
    if M:
        cuda_ext().quant_mxf8_act(xq, sfa, x)
        _LAUNCHES[0] += 1
    return xq, sfa


def rms_norm_mxf8(x: torch.Tensor, w: torch.Tensor, eps: float, offset: float = 0.0,
                  residual: Optional[torch.Tensor] = None):
    """RMSNorm (residual += x first when given, in place) emitting the MXFP8
    GEMM operand directly: (e4m3 [M, H], UE8M0 scale chunks)."""
    M, H = x.shape
    xq = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=x.device)
    sfa = torch.empty((M + 127) // 128, H // 128, 512, dtype=torch.uint8, device=x.device)
    if M:
        cuda_ext().rms_norm_mxf8(xq, sfa, x.contiguous(), residual, w, eps, offset)
        _LAUNCHES[0] += 1
    return xq, sfa


def linear_mxf8_q(xq: torch.Tensor, sfa: torch.Tensor, wq: torch.Tensor, wsf: torch.Tensor,
                  bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                  silu_mul: bool = False, act: str = "silu") -> torch.Tensor:
    """MXFP8 GEMM on an already quantised operand (e.g. from rms_norm_mxf8); with
    silu_mul the gated epilogue applies `act` (SiLU or GELU-tanh) to the gate."""
    M, N = xq.shape[0], wq.shape[0]
    out = torch.empty(M, N // 2 if silu_mul else N, dtype=torch.bfloat16, device=xq.device)
    if M:
        epi = (1 | _gate(act)) if silu_mul else 0
        _LAUNCHES[0] += cuda_ext().gemm_mxf8(out, xq, sfa, wq, wsf, bias, residual, epi, 0, 0)
    return out


def linear_mxf8_silu_q(xq: torch.Tensor, sfa: torch.Tensor, wq: torch.Tensor, wsf: torch.Tensor,
                       bias: Optional[torch.Tensor] = None, act: str = "silu"):
    """gate/up MXFP8 GEMM (rows interleaved in 64-row blocks) whose epilogue
    emits act(gate)*up directly as the next MXFP8 operand (e4m3 + scales)."""
    M, N = xq.shape[0], wq.shape[0]
    q = torch.empty(M, N // 2, dtype=torch.float8_e4m3fn, device=xq.device)
    sf = torch.empty((M + 127) // 128, N // 256, 512, dtype=torch.uint8, device=xq.device)
    if M:
        _LAUNCHES[0] += cuda_ext().gemm_mxf8_silu_q(q, sf, xq, sfa, wq, wsf, bias, _gate(act) >> 8)
    return q, sf


def linear_fp8(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
               bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
               silu_mul: bool = False, wsf: Optional[torch.Tensor] = None, act: str = "silu") -> torch.Tensor:
    """Block-scaled fp8 GEMM: x bf16 [M,K] is quantised 1x128 on the fly (one
    kernel), wq e4m3 [N,K] carries fp32 128x128 scales ws [N/128, K/128].
    With `wsf` (the same scales as power-of-two UE8M0 chunks) the GEMM applies
    the scales inside the tensor-core MMA (kind::mxf8f6f4.block_scale);
    without it, fp32 scales are applied per 128-K block in the epilogue.
    With silu_mul the weight rows are gate/up interleaved in 64-row blocks and
    the output is act(gate) * up with N/2 columns (act: SiLU or GELU-tanh)."""
    M, N = x.shape[0], wq.shape[0]
    n_out = N // 2 if silu_mul else N
    if not x.is_cuda:
        if wsf is not None:
            xq, xs_r = ref.quant_mxf8_act(x)
            y = ref.fp8_block_gemm(xq, xs_r, wq, ws)
        else:
            xq, xs = quant_fp8_act(x)
            y = ref.fp8_block_gemm(xq, xs.t(), wq, ws)
        if bias is not None:
            y = y + bias.float()
        if silu_mul:
            v = y.view(M, N // 128, 2, 64)
            g = (torch.nn.functional.silu(v[:, :, 0]) if _gate(act) == 0
                 else torch.nn.functional.gelu(v[:, :, 0], approximate="tanh"))
            y = (g * v[:, :, 1]).reshape(M, n_out)
        if residual is not None:
            y = y + residual.float()
        return y.to(x.dtype)
    out = torch.empty(M, n_out, dtype=torch.bfloat16, device=x.device)
    if M == 0:
        return out
    if wsf is not None:
        xq, sfa = quant_mxf8_act(x)
        epi = (1 | _gate(act)) if silu_mul else 0
        _LAUNCHES[0] += cuda_ext().gemm_mxf8(out, xq, sfa, wq, wsf, bias, residual, epi, 0, 0)
        return out
    xq, xs = quant_fp8_act(x)
    if silu_mul and _gate(act):
        # the fp32-scale kernel's gated epilogue is SiLU: GELU gates run on the full output
        y = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
        _LAUNCHES[0] += cuda_ext().gemm_fp8_block(y, xq, xs, wq, ws, bias, residual, 0, 0)
        return _act_mul_interleaved(y, act)
    _LAUNCHES[0] += cuda_ext().gemm_fp8_block(out, xq, xs, wq, ws, bias, residual, 1 if silu_mul else 0, 0)
    return out


# ----------------------------------------------------------------------------- MoE
def moe_forward(h: torch.Tensor, router: torch.Tensor, w13_il: torch.Tensor, w2: torch.Tensor, topk: int,
                e_lo: int = 0, renormalize: bool = True,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Routed MoE block over the local experts [e_lo, e_lo + w13_il.shape[0]):
    fused router + top-k softmax, expert-sorted gather (128-aligned segments),
    grouped tcgen05 GEMMs (gate/up with SiLU epilogue, then down) and the
    weighted combine; no host synchronisation.  Tokens routed to experts of
    other ranks contribute zero (the caller sums partial outputs over ranks)."""
    out = torch.empty_like(h)
    if h.shape[0] == 0:
        return out
    _LAUNCHES[0] += cuda_ext().moe_forward(out, h.contiguous(), router, w13_il, w2, topk, e_lo, renormalize,
                                          residual)
    return out


def interleave_gate_up_experts(w13: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[E, 2I, K] per-expert [gate | up] rows -> the 64-row interleaved layout."""
    return torch.stack([interleave_gate_up(w13[e], block) for e in range(w13.shape[0])]).contiguous()


# ----------------------------------------------------------------------------- sampling
def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           min_p: torch.Tensor, seeds: torch.Tensor, offsets: torch.Tensor, greedy_all: bool,
           want_logprobs: bool = False):
    """Returns (token ids int64 [B], logprob of the chosen token fp32 [B])."""
    C = cuda_ext()
    B, V = logits.shape
    tokens = torch.empty(B, dtype=torch.int64, device=logits.device)
    lp = torch.empty(B, dtype=torch.float32, device=logits.device)
    if greedy_all:
        z = _greedy_params(B, logits.device)
        C.sample_rows(tokens, lp, logits, *z)
    else:
        C.sample_rows(tokens, lp, logits, temperature, top_k, top_p, min_p, seeds, offsets)
    _LAUNCHES[0] += 1
    return tokens, lp


_GREEDY: dict = {}


def _greedy_params(B: int, device) -> tuple:
    """Per-row parameter vectors of an all-greedy batch (temperature 0), cached by size."""
    key = (B, str(device))
    z = _GREEDY.get(key)
    if z is None:
        f = torch.zeros(B, dtype=torch.float32, device=device)
        i = torch.zeros(B, dtype=torch.int32, device=device)
        l = torch.zeros(B, dtype=torch.int64, device=device)
        z = _GREEDY[key] = (f, i, f, f, l, l)
    return z


def sample_slots(logits: torch.Tensor, row_info: torch.Tensor, tables) -> tuple:
    """Samples every row with the parameters of its device slot (`engine.sampler.SlotTable`):
    penalties, logit bias and min_tokens applied in the kernel, which then advances the
    slot's generated-token counter and penalty counts.  Returns (ids int64 [R], logprob fp32 [R])."""
    B = logits.shape[0]
    tokens = torch.empty(B, dtype=torch.int64, device=logits.device)
    lp = torch.empty(B, dtype=torch.float32, device=logits.device)
    cuda_ext().sample_slots(tokens, lp, logits, row_info, list(tables))
    _LAUNCHES[0] += 1
    return tokens, lp
