"""Plain PyTorch fp32 restatements of every device op.

These are the oracles for the sm_100a kernels (tests compare the CUDA output
to these) and the CPU execution path of the engine (the tiny-Llama CPU
configuration runs entirely on them).  Math follows the reference's CPU code:
RMSNorm with fp32 accumulation (crates/rusteeze-model/src/architectures/
common.rs:33-45), neox rotate-half RoPE (common.rs:142-170), SwiGLU MLP
(common.rs:354-361), GQA attention with online-softmax semantics
(crates/rusteeze-engine/src/flash_attention.rs:186-318), and the sampler
pipeline penalties -> temperature -> top-k -> top-p (crates/rusteeze-engine/
src/sampler.rs:56-244, simd_ops.rs:89-119).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

BLOCK_SIZE = 16


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, offset: float = 0.0) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps) * (w.float() + offset)).to(x.dtype)


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                       offset: float = 0.0) -> Tuple[torch.Tensor, torch.Tensor]:
    """residual <- x + residual ; returns (rms_norm(residual), residual)."""
    r = (x.float() + residual.float()).to(residual.dtype)
    return rms_norm(r, w, eps, offset), r


def layer_norm(x, w, b, eps):
    return F.layer_norm(x.float(), (x.shape[-1],), w.float(), None if b is None else b.float(), eps).to(x.dtype)


def rope_cos_sin_cache(head_dim: int, max_pos: int, theta: float, scaling=None,
                       device=None) -> torch.Tensor:
    """Returns [max_pos, head_dim] fp32: first half cos, second half sin."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float64)
    if scaling is not None and scaling.type == "linear":
        pos = pos / scaling.factor
    elif scaling is not None and scaling.type == "llama3":
        # Llama-3.1 frequency-dependent scaling of the inverse frequencies.
        factor = scaling.factor
        lo = scaling.low_freq_factor or 1.0
        hi = scaling.high_freq_factor or 4.0
        old = scaling.original_max_position_embeddings or 8192
        lo_wl, hi_wl = old / lo, old / hi
        wl = 2 * math.pi / inv
        smooth = (old / wl - lo) / (hi - lo)
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
    elif scaling is not None and scaling.type == "dynamic":
        base = theta * ((scaling.factor * max_pos / (scaling.original_max_position_embeddings or max_pos))
                        - (scaling.factor - 1)) ** (head_dim / (head_dim - 2))
        inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    freqs = torch.outer(pos, inv)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1).float().to(device)


def identity_cos_sin(head_dim: int, max_pos: int, device=None) -> torch.Tensor:
    """The cos/sin table of a zero rotation (cos 1, sin 0): models without RoPE (ALiBi)
    run the fused RoPE + KV-write kernel with it, which then only writes the cache."""
    t = torch.zeros(max_pos, head_dim, dtype=torch.float32, device=device)
    t[:, : head_dim // 2] = 1.0
    return t


def alibi_slopes(num_heads: int) -> torch.Tensor:
    """ALiBi head slopes (Press et al., "Train Short, Test Long", 2022): for n a power of
    two, head i (1-based) gets 2^(-8 i / n).  Otherwise the n' = 2^floor(log2 n) slopes of
    that geometric sequence come first, followed by the odd-indexed terms 2^(-8 (2j - 1) /
    (2 n')), j = 1, 2, ... of the sequence for 2 n' heads (the interleaving the paper's
    reference code uses).  The reference library's `get_alibi_slopes`
    (crates/rusteeze-tensor/src/attention.rs:342-368) agrees for powers of two."""
    def geometric(n: int):
        return [2.0 ** (-8.0 * i / n) for i in range(1, n + 1)]
    p = 1 << (max(1, num_heads).bit_length() - 1)
    slopes = geometric(p)
    if p < num_heads:
        slopes += [2.0 ** (-8.0 * (2 * j - 1) / (2 * p)) for j in range(1, num_heads - p + 1)]
    return torch.tensor(slopes, dtype=torch.float32)


def alibi_bias(slopes: torch.Tensor, q_pos: torch.Tensor, k_pos: torch.Tensor) -> torch.Tensor:
    """[H, q, k] additive logit bias slope_h * (k_pos - q_pos): 0 on the diagonal, more
    negative the further back the key."""
    rel = (k_pos.view(1, -1) - q_pos.view(-1, 1)).float()
    return slopes.float().view(-1, 1, 1) * rel.unsqueeze(0)


def rope(q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor):
    """Neox (rotate-half) RoPE, in place on q [T,Hq,D] and k [T,Hkv,D]."""
    d = q.shape[-1]
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, : d // 2].unsqueeze(1), cs[:, d // 2:].unsqueeze(1)

    def apply(x):
        xf = x.float()
        x1, x2 = xf[..., : d // 2], xf[..., d // 2:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)

    q.copy_(apply(q))
    k.copy_(apply(k))
    return q, k


FP8_KV_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2)


def is_fp8(dtype: torch.dtype) -> bool:
    return dtype in FP8_KV_DTYPES


def to_kv(x: torch.Tensor, dtype: torch.dtype, scale: float = 1.0) -> torch.Tensor:
    """Cache encoding: bf16/f16/f32 as is; fp8 holds x / scale rounded to nearest even and
    saturated to the largest finite value (448 for e4m3, 57344 for e5m2), NaN kept."""
    if not is_fp8(dtype):
        return x.to(dtype)
    m = torch.finfo(dtype).max
    y = x.float() / scale
    return torch.where(torch.isnan(y), y, y.clamp(-m, m)).to(dtype)


def reshape_and_cache(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      slot_mapping: torch.Tensor, k_scale: float = 1.0, v_scale: float = 1.0) -> None:
    """k,v: [T, Hkv, D]; caches: [num_blocks, Hkv, BLOCK, D]; slot<0 is skipped."""
    sm = slot_mapping.long()
    keep = sm >= 0
    sm = sm[keep]
    blk, off = sm // BLOCK_SIZE, sm % BLOCK_SIZE
    k_cache[blk, :, off, :] = to_kv(k[keep], k_cache.dtype, k_scale)
    v_cache[blk, :, off, :] = to_kv(v[keep], v_cache.dtype, v_scale)


def silu_mul(x: torch.Tensor) -> torch.Tensor:
    """x: [T, 2I] laid out [gate | up] -> silu(gate) * up."""
    g, u = x.float().chunk(2, dim=-1)
    return (F.silu(g) * u).to(x.dtype)


def gelu_tanh_mul(x: torch.Tensor) -> torch.Tensor:
    g, u = x.float().chunk(2, dim=-1)
    return (F.gelu(g, approximate="tanh") * u).to(x.dtype)


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype)


def gather_kv(cache: torch.Tensor, block_table: torch.Tensor, seq_len: int) -> torch.Tensor:
    """cache [nb, Hkv, BLOCK, D] -> [seq_len, Hkv, D] for one sequence (fp8 caches are
    gathered as bytes and keep their dtype)."""
    nblk = (seq_len + BLOCK_SIZE - 1) // BLOCK_SIZE
    src = cache.view(torch.uint8) if is_fp8(cache.dtype) else cache
    blocks = src[block_table[:nblk].long()]                   # [nblk, Hkv, BLOCK, D]
    if src is not cache:
        blocks = blocks.view(cache.dtype)
    return blocks.permute(0, 2, 1, 3).reshape(-1, cache.shape[1], cache.shape[3])[:seq_len]


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    query_start_loc: torch.Tensor, seq_lens: torch.Tensor, block_tables: torch.Tensor,
                    scale: float, sliding_window: Optional[int] = None,
                    softcap: Optional[float] = None,
                    alibi: Optional[torch.Tensor] = None, k_scale: float = 1.0,
                    v_scale: float = 1.0) -> torch.Tensor:
    """Varlen causal GQA attention over a paged KV cache.

    q: [T, Hq, D]; sequence i owns query rows query_start_loc[i]:query_start_loc[i+1],
    which are the LAST q_len positions of its seq_lens[i]-long context.  alibi: [Hq]
    slopes, added as slope * (k_pos - q_pos) after the soft-cap.  fp8 caches hold
    k / k_scale and v / v_scale.
    """
    out = torch.empty_like(q)
    hq, hkv = q.shape[1], k_cache.shape[1]
    g = hq // hkv
    qsl = query_start_loc.tolist()
    for i, L in enumerate(seq_lens.tolist()):
        a, b = qsl[i], qsl[i + 1]
        ql = b - a
        if ql == 0:
            continue
        K = (gather_kv(k_cache, block_tables[i], L).float() * k_scale).repeat_interleave(g, dim=1)  # [L,Hq,D]
        V = (gather_kv(v_cache, block_tables[i], L).float() * v_scale).repeat_interleave(g, dim=1)
        Q = q[a:b].float()
        s = torch.einsum("qhd,khd->hqk", Q, K) * scale
        if softcap:
            s = softcap * torch.tanh(s / softcap)
        qpos = torch.arange(L - ql, L).unsqueeze(1)
        kpos = torch.arange(L).unsqueeze(0)
        if alibi is not None:
            s = s + alibi_bias(alibi.cpu(), qpos.view(-1), kpos.view(-1)).to(s.device)
        mask = kpos > qpos
        if sliding_window:
            mask |= kpos <= qpos - sliding_window
        s = s.masked_fill(mask.unsqueeze(0), float("-inf"))
        p = torch.softmax(s, dim=-1)
        out[a:b] = torch.einsum("hqk,khd->qhd", p, V).to(q.dtype)
    return out


# ----------------------------------------------------------------------------- sampling
def apply_penalties(logits: torch.Tensor, output_tokens: list, prompt_tokens: list,
                    rep: torch.Tensor, freq: torch.Tensor, pres: torch.Tensor) -> torch.Tensor:
    """Repetition penalty over prompt+output tokens (divide positive, multiply
    negative logits), then frequency/presence penalties over output tokens."""
    logits = logits.clone()
    for i in range(logits.shape[0]):
        seen = set(prompt_tokens[i]) | set(output_tokens[i])
        if rep[i] != 1.0 and seen:
            idx = torch.tensor(sorted(seen), dtype=torch.long)
            v = logits[i, idx]
            logits[i, idx] = torch.where(v > 0, v / rep[i], v * rep[i])
        if output_tokens[i] and (freq[i] != 0.0 or pres[i] != 0.0):
            cnt = torch.bincount(torch.tensor(output_tokens[i], dtype=torch.long),
                                 minlength=logits.shape[1]).float()
            logits[i] -= freq[i] * cnt + pres[i] * (cnt > 0).float()
    return logits


def topk_topp_minp_probs(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                         top_p: torch.Tensor, min_p: torch.Tensor) -> torch.Tensor:
    """Filtered, renormalised probabilities per row (temperature > 0 rows)."""
    x = logits.float() / temperature.clamp_min(1e-5).unsqueeze(1)
    probs = torch.softmax(x, dim=-1)
    V = x.shape[1]
    sp, si = probs.sort(dim=-1, descending=True)
    ranks = torch.arange(V).unsqueeze(0)
    k = torch.where(top_k > 0, top_k, torch.full_like(top_k, V)).unsqueeze(1)
    keep = ranks < k
    cum = sp.cumsum(-1) - sp                       # mass strictly before this token
    keep &= cum < top_p.unsqueeze(1)
    keep &= sp >= (min_p.unsqueeze(1) * sp[:, :1])
    keep[:, 0] = True
    sp = torch.where(keep, sp, torch.zeros_like(sp))
    out = torch.zeros_like(probs).scatter(1, si, sp)
    return out / out.sum(-1, keepdim=True)


def spec_verify_greedy(draft_tokens: torch.Tensor, target_argmax: torch.Tensor):
    """draft [B,k], target_argmax [B,k+1] -> (accepted count [B], emitted tokens [B,k+1])."""
    B, k = draft_tokens.shape
    match = (draft_tokens == target_argmax[:, :k]).int()
    acc = match.cumprod(dim=1).sum(dim=1)
    out = torch.full((B, k + 1), -1, dtype=torch.long)
    for b in range(B):
        n = int(acc[b])
        out[b, :n] = draft_tokens[b, :n]
        out[b, n] = target_argmax[b, n]
    return acc, out


# ----------------------------------------------------------------------------- fp8
FP8_E4M3_MAX = 448.0


def quant_fp8_act(x: torch.Tensor, group: int = 128):
    """1 x group activation quant: x [M, K] -> (q e4m3 [M,K], scales fp32 [M, K/group])."""
    M, K = x.shape
    xg = x.float().view(M, K // group, group)
    amax = xg.abs().amax(-1).clamp_min(1e-12)
    s = amax / FP8_E4M3_MAX
    q = (xg / s.unsqueeze(-1)).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(M, K), s


def quant_fp8_weight(w: torch.Tensor, block: int = 128):
    """128x128 block weight quant: w [N, K] -> (q [N,K] e4m3, scales fp32 [ceil(N/b), K/b])."""
    N, K = w.shape
    nb = (N + block - 1) // block
    wp = torch.zeros(nb * block, K, dtype=torch.float32, device=w.device)
    wp[:N] = w.float()
    wb = wp.view(nb, block, K // block, block)
    amax = wb.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    s = amax / FP8_E4M3_MAX
    q = (wb / s[:, None, :, None]).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(nb * block, K)[:N].contiguous(), s


def pow2_ceil(s: torch.Tensor) -> torch.Tensor:
    """Smallest power of two >= s (s > 0): the UE8M0 scale of a block."""
    m, e = torch.frexp(s)
    e = torch.where(m == 0.5, e - 1, e)
    return torch.ldexp(torch.ones_like(s), e.clamp(-126, 126))


def quant_mxf8_act(x: torch.Tensor, group: int = 128):
    """1 x group activation quant with power-of-two (UE8M0) scales:
    x [M, K] -> (q e4m3 [M, K], scales fp32 [M, K/group])."""
    M, K = x.shape
    xg = x.float().view(M, K // group, group)
    amax = xg.abs().amax(-1)
    s = torch.where(amax > 0, pow2_ceil((amax / FP8_E4M3_MAX).clamp_min(1e-38)), torch.ones_like(amax))
    q = (xg / s.unsqueeze(-1)).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(M, K), s


def quant_mxf8_weight(w: torch.Tensor, block: int = 128):
    """128x128 block weight quant with power-of-two scales: w [N, K] ->
    (q [N, K] e4m3, scales fp32 [ceil(N/b), K/b])."""
    N, K = w.shape
    nb = (N + block - 1) // block
    wp = torch.zeros(nb * block, K, dtype=torch.float32, device=w.device)
    wp[:N] = w.float()
    wb = wp.view(nb, block, K // block, block)
    amax = wb.abs().amax(dim=(1, 3))
    s = torch.where(amax > 0, pow2_ceil((amax / FP8_E4M3_MAX).clamp_min(1e-38)), torch.ones_like(amax))
    q = (wb / s[:, None, :, None]).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)
    return q.view(nb * block, K)[:N].contiguous(), s


def pack_block_scales_ue8m0(s: torch.Tensor) -> torch.Tensor:
    """fp32 power-of-two scales of 128x128 blocks [R/128, K/128] -> the GEMM's
    scale chunks: uint8 [R/128, K/128, 512], every byte of a chunk the block's
    biased exponent (one scale per 128 rows x 32 K-elements, all equal)."""
    _, e = torch.frexp(s)                       # s = 0.5 * 2^e  ->  log2(s) = e - 1
    byte = (e - 1 + 127).clamp(1, 254).to(torch.uint8)
    return byte.unsqueeze(-1).expand(*s.shape, 512).contiguous()


def pack_act_scales_ue8m0(s: torch.Tensor) -> torch.Tensor:
    """fp32 power-of-two 1x128 scales [M, K/128] -> chunks [ceil(M/128), K/128, 512]:
    row r of a 128-row block keeps its 4 K-chunk bytes at (r%32)*16 + (r/32)*4;
    rows past M get the neutral byte 127 (scale 1)."""
    M, kb = s.shape
    mb = (M + 127) // 128
    _, e = torch.frexp(s)
    byte = (e - 1 + 127).clamp(1, 254).to(torch.uint8)
    full = torch.full((mb * 128, kb), 127, dtype=torch.uint8, device=s.device)
    full[:M] = byte
    # [mb, r1(4), r0(32), kb] -> [mb, kb, r0, r1, kc(4)]
    t = full.view(mb, 4, 32, kb).permute(0, 3, 2, 1).unsqueeze(-1).expand(mb, kb, 32, 4, 4)
    return t.reshape(mb, kb, 512).contiguous()


def unpack_act_scales_ue8m0(sfa: torch.Tensor, M: int, K: int) -> torch.Tensor:
    """Inverse of the activation scale layout: chunks [ceil(M/128), K/128, 512]
    -> fp32 scales [M, K/128] (the K-chunk-0 byte of every row)."""
    kb = K // 128
    ch = sfa.view(-1, kb, 512).to(torch.int32)
    r = torch.arange(M, device=sfa.device)
    off = (r % 128 % 32) * 16 + (r % 128 // 32) * 4
    e = ch[r // 128].gather(2, off.view(M, 1, 1).expand(M, kb, 1)).squeeze(-1)
    return torch.ldexp(torch.ones(M, kb, device=sfa.device), e - 127)


def fp8_block_gemm(xq, xs, wq, ws, block: int = 128):
    """Dequantise-then-matmul oracle of the block-scaled fp8 GEMM."""
    M, K = xq.shape
    N = wq.shape[0]
    x = xq.float().view(M, K // block, block) * xs.unsqueeze(-1)
    nb = ws.shape[0]
    wp = torch.zeros(nb * block, K, device=wq.device)
    wp[:N] = wq.float()
    w = (wp.view(nb, block, K // block, block) * ws[:, None, :, None]).view(nb * block, K)[:N]
    return x.view(M, K) @ w.t()


# ----------------------------------------------------------------------------- moe
def moe_topk_softmax(router_logits: torch.Tensor, k: int):
    """Mixtral routing: top-k over softmax, weights renormalised over the k."""
    p = torch.softmax(router_logits.float(), dim=-1)
    w, idx = p.topk(k, dim=-1)
    w = w / w.sum(-1, keepdim=True)
    return w, idx
