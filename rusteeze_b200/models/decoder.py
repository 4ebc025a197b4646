"""One decoder-only transformer covering the whole model zoo.

Architectures (crates/rusteeze-model/src/config.rs:15-62 enumerates them; the
reference implements only Llama (architectures/llama.rs:86-339) and Mistral
(architectures/mistral.rs:178-586)):

  llama / mistral  pre-norm RMSNorm, GQA attention with neox RoPE, SwiGLU MLP;
                   Mistral adds a sliding window (mistral.rs:334-363), applied
                   inside the attention kernel instead of as a host mask.
  qwen2            llama + bias on the fused QKV projection.
  phi3             llama layout; its checkpoints already store fused qkv_proj
                   and gate_up_proj tensors.
  mixtral          llama attention + top-2 softmax-routed sparse MoE of SwiGLU
                   experts (absent from the reference).
  gemma            (1 + w) RMSNorm, sqrt(hidden) embedding scale, GeGLU (tanh).
  gemma2           gemma + sandwich norms around attention and MLP, attention
                   and final-logit soft-capping, local/global alternating
                   sliding window, query_pre_attn_scalar.

The forward works on a flattened token batch (continuous batching): tokens of
all sequences are concatenated; `AttentionMetadata` says which rows belong to
which sequence and where their K/V live in the paged cache.

Weights are stored fused and K-major for the GEMM kernel: qkv [(Hq+2Hkv)*D, H],
gate_up [2I, H] as [gate | up], o [H, Hq*D], down [H, I].  Under tensor
parallelism every rank holds its own slice (column split of qkv/gate_up by
head/column, row split of o/down, vocab split of embedding and LM head).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn as nn

from rusteeze_b200 import ops
from rusteeze_b200.utils.op_timer import OP_TIMER
from rusteeze_b200.core.types import ModelArchitecture
from rusteeze_b200.models.config import ModelConfig
from rusteeze_b200.ops import reference as ref


@dataclass
class AttentionMetadata:
    """Flattened-batch attention description for one forward.

    Sequences [0, num_decode_seqs) are single-token decodes occupying token
    rows [0, num_decode_seqs); the rest are prefill (or multi-token verify)
    chunks.  For sequence i, its query rows are query_start_loc[i] :
    query_start_loc[i+1] and they are the LAST rows of a seq_lens[i]-long
    context whose KV pages are block_tables[i, :]."""
    num_seqs: int
    num_tokens: int
    num_decode_seqs: int
    query_start_loc: torch.Tensor          # int32 [S+1]
    seq_lens: torch.Tensor                 # int32 [S]
    block_tables: torch.Tensor             # int32 [S, max_blocks]
    slot_mapping: torch.Tensor             # int64 [T]  (-1: do not write)
    max_query_len: int = 1
    max_seq_len: int = 0
    decode_num_splits: int = 1
    decode_workspace: Optional[torch.Tensor] = None
    # rows of the hidden state whose logits are needed (last token of each seq,
    # or every verify position for speculative decoding)
    logits_indices: Optional[torch.Tensor] = None
    # KV blocks of the non-decode sequences (sum of ceil(seq_len / 16) over [num_decode_seqs,
    # num_seqs)): the size of the bf16 scratch an fp8 cache is gathered into for prefill
    prefill_kv_blocks: int = 0


class TPGroup:
    """Tensor-parallel context handed to the model.  Single-GPU default is a
    no-op; `rusteeze_b200.parallel.tp.TPComm` implements the real one."""
    rank = 0
    size = 1

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def all_gather_last_dim(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def row_parallel_linear(self, x, w, bias=None):
        """GEMM whose output must be summed over ranks (o_proj / down_proj)."""
        return self.all_reduce(ops.linear(x, w, bias))


def _split(n: int, size: int, rank: int):
    assert n % size == 0, f"dimension {n} not divisible by tensor-parallel size {size}"
    per = n // size
    return rank * per, (rank + 1) * per


class DecoderLM(nn.Module):
    def __init__(self, cfg: ModelConfig, dtype=torch.bfloat16, device="cpu",
                 tp: Optional[TPGroup] = None, ep_rank: int = 0, ep_size: int = 1):
        super().__init__()
        self.cfg = cfg
        self.tp = tp or TPGroup()
        self.dtype = dtype
        self.device = torch.device(device)
        tps, tpr = self.tp.size, self.tp.rank
        self.ep_rank, self.ep_size = ep_rank, ep_size
        H, D = cfg.hidden_size, cfg.head_dim
        assert cfg.num_attention_heads % tps == 0, "q heads must divide by TP size"
        self.hq = cfg.num_attention_heads // tps
        # KV heads are split when possible, replicated otherwise (e.g. 8 kv heads at TP16)
        self.hkv = max(1, cfg.num_key_value_heads // tps)
        self.inter = cfg.intermediate_size // tps if not cfg.is_moe else cfg.intermediate_size
        self.vocab_lo, self.vocab_hi = _split(_pad_vocab(cfg.vocab_size, tps), tps, tpr)
        arch = cfg.architecture
        self.is_gemma = arch in (ModelArchitecture.GEMMA, ModelArchitecture.GEMMA2)
        self.is_gemma2 = arch == ModelArchitecture.GEMMA2
        self.act = "gelu_tanh" if (self.is_gemma or "gelu" in cfg.hidden_act) else "silu"
        e = lambda *s: torch.empty(*s, dtype=dtype, device=device)  # noqa: E731

        self.embed = nn.Parameter(e(self.vocab_hi - self.vocab_lo, H), requires_grad=False)
        self.layers = nn.ModuleList()
        for li in range(cfg.num_hidden_layers):
            L = nn.Module()
            L.input_norm = nn.Parameter(e(H), requires_grad=False)
            L.post_attn_norm = nn.Parameter(e(H), requires_grad=False)
            L.qkv = nn.Parameter(e((self.hq + 2 * self.hkv) * D, H), requires_grad=False)
            L.qkv_bias = (nn.Parameter(e((self.hq + 2 * self.hkv) * D), requires_grad=False)
                          if cfg.attention_bias else None)
            L.o = nn.Parameter(e(H, self.hq * D), requires_grad=False)
            if self.is_gemma2:
                L.pre_ff_norm = nn.Parameter(e(H), requires_grad=False)
                L.post_ff_norm = nn.Parameter(e(H), requires_grad=False)
            if cfg.is_moe:
                E = cfg.num_local_experts
                assert E % ep_size == 0, "experts must divide by EP size"
                self.e_lo, self.e_hi = _split(E, ep_size, ep_rank)
                ne = self.e_hi - self.e_lo
                L.router = nn.Parameter(e(E, H), requires_grad=False)
                L.w13 = nn.Parameter(e(ne, 2 * cfg.intermediate_size, H), requires_grad=False)
                L.w2 = nn.Parameter(e(ne, H, cfg.intermediate_size), requires_grad=False)
            else:
                L.gate_up = nn.Parameter(e(2 * self.inter, H), requires_grad=False)
                L.down = nn.Parameter(e(H, self.inter), requires_grad=False)
            L.sliding_window = cfg.layer_sliding_window(li)
            self.layers.append(L)
        self.norm = nn.Parameter(e(H), requires_grad=False)
        self.lm_head = (None if cfg.tie_word_embeddings
                        else nn.Parameter(e(self.vocab_hi - self.vocab_lo, H), requires_grad=False))
        if cfg.use_alibi:
            # no rotation: the fused RoPE + KV-write kernel runs with a zero-angle table (a
            # plain cache write) and the attention kernels add slope * (k_pos - q_pos); this
            # rank's query heads are [tpr * hq, (tpr + 1) * hq)
            self.register_buffer("cos_sin", ref.identity_cos_sin(D, cfg.max_position_embeddings, device=device),
                                 persistent=False)
            self.register_buffer("alibi", ref.alibi_slopes(cfg.num_attention_heads)[
                tpr * self.hq:(tpr + 1) * self.hq].contiguous().to(device), persistent=False)
        else:
            self.register_buffer("cos_sin", ref.rope_cos_sin_cache(
                D, cfg.max_position_embeddings, cfg.rope_theta, cfg.rope_scaling, device=device),
                persistent=False)
            self.alibi = None
        self.moe_impl = None   # set by parallel.moe for EP / fused dispatch
        # an fp8 KV cache holds k / k_scale and v / v_scale (1.0: the values as they are,
        # saturated at the format's largest finite value)
        self.kv_scales = (1.0, 1.0)

    # ------------------------------------------------------------------ helpers
    @property
    def lm_head_weight(self) -> torch.Tensor:
        return self.embed if self.lm_head is None else self.lm_head

    def embed_tokens(self, ids: torch.Tensor) -> torch.Tensor:
        """Embedding rows (vocab-parallel at TP > 1: each rank gathers the rows of its
        vocabulary shard and zeros elsewhere, one kernel with Gemma's scale folded in, and
        the ranks' rows are summed)."""
        h = ops.embedding(ids, self.embed, self.vocab_lo, self.cfg.vocab_size, self.cfg.embed_scale)
        if self.tp.size > 1:
            h = self.tp.all_reduce(h)
        return h

    def _lin(self, x: torch.Tensor, owner, name: str, bias=None) -> torch.Tensor:
        q = getattr(owner, name + "_q", None)
        if q is not None:
            return ops.linear_fp8(x, q, getattr(owner, name + "_s"), bias, wsf=getattr(owner, name + "_sf", None))
        return ops.linear(x, getattr(owner, name), bias)

    def _row_parallel(self, x: torch.Tensor, owner, name: str) -> torch.Tensor:
        q = getattr(owner, name + "_q", None)
        if q is not None:
            return self.tp.all_reduce(ops.linear_fp8(x, q, getattr(owner, name + "_s"),
                                                     wsf=getattr(owner, name + "_sf", None)))
        return self.tp.row_parallel_linear(x, getattr(owner, name))

    def _mlp(self, L, h: torch.Tensor) -> torch.Tensor:
        if getattr(L, "gate_up_q", None) is not None:
            a = ops.linear_fp8(h, L.gate_up_q, L.gate_up_s, silu_mul=True, wsf=getattr(L, "gate_up_sf", None),
                               act=self.act)
            return self._row_parallel(a, L, "down")
        if getattr(L, "gate_up_il", None) is not None and h.is_cuda:
            # act(gate)*up fused in the GEMM epilogue (SwiGLU, or Gemma's GeGLU)
            a = ops.linear_silu_mul(h, L.gate_up_il, act=self.act)
        else:
            gu = ops.linear(h, L.gate_up)
            a = ops.silu_mul(gu) if self.act == "silu" else ops.gelu_tanh_mul(gu)
        return self.tp.row_parallel_linear(a, L.down)

    @torch.no_grad()
    def prepare_for_gpu(self) -> None:
        """Re-lays weights for the GPU kernels: gate/up rows interleaved in
        64-row blocks for the fused gated epilogue, SiLU or GELU-tanh (the
        [gate | up] copy is dropped to save HBM)."""
        if not self.device.type == "cuda" or getattr(self, "fp8", False):
            return
        if self.cfg.is_moe:
            if self.act != "silu":
                return
            if self.cfg.intermediate_size % 64 or self.cfg.hidden_size % 256:
                return
            for L in self.layers:
                if getattr(L, "w13_il", None) is not None:
                    continue
                L.w13_il = ops.interleave_gate_up_experts(L.w13)
                L.w13 = nn.Parameter(torch.empty(0, dtype=self.dtype, device=self.device), requires_grad=False)
            return
        if self.inter % 64:
            return
        for L in self.layers:
            if getattr(L, "gate_up_il", None) is not None:
                continue
            L.gate_up_il = ops.interleave_gate_up(L.gate_up)
            L.gate_up = nn.Parameter(torch.empty(0, dtype=self.dtype, device=self.device), requires_grad=False)

    def _moe(self, L, h: torch.Tensor) -> torch.Tensor:
        if self.moe_impl is not None:
            return self.moe_impl(L, h)
        if getattr(L, "w13_il", None) is not None and h.is_cuda:
            out = ops.moe_forward(h, L.router, L.w13_il, L.w2, self.cfg.num_experts_per_tok, self.e_lo,
                                  True)
            return self.tp.all_reduce(out) if self.tp.size > 1 else out
        return moe_forward_local(L, h, self.cfg, self.e_lo, self.e_hi, self.tp)

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, meta: AttentionMetadata,
                kv_caches: List[torch.Tensor]) -> torch.Tensor:
        if self._fused_tp_ok(input_ids.shape[0]):
            return self._forward_fused_tp(input_ids, positions, meta, kv_caches)
        cfg = self.cfg
        eps, off = cfg.rms_norm_eps, cfg.norm_offset
        D = cfg.head_dim
        sec = OP_TIMER.section
        with sec("embed"):
            h = self.embed_tokens(input_ids)
        residual = None
        # MXFP8 weights: the norms emit the GEMM operand (e4m3 + UE8M0 scales) directly
        mx = h.is_cuda and getattr(self, "fp8_format", None) == "ue8m0" and not self.is_gemma2
        for li, L in enumerate(self.layers):
            kv = kv_caches[li]
            if mx:
                with sec("norm_ag"):
                    if residual is None:
                        residual = h
                        xq = ops.rms_norm_mxf8(h, L.input_norm, eps, off)
                    else:
                        xq = ops.rms_norm_mxf8(h, L.input_norm, eps, off, residual=residual)
                with sec("qkv_gemm"):
                    qkv = ops.linear_mxf8_q(*xq, L.qkv_q, L.qkv_sf, L.qkv_bias)
            else:
                with sec("norm_ag"):
                    if residual is None:
                        residual = h
                        x = ops.rms_norm(h, L.input_norm, eps, off)
                    else:
                        x, residual = ops.fused_add_rms_norm(h, residual, L.input_norm, eps, off)
                with sec("qkv_gemm"):
                    qkv = self._lin(x, L, "qkv", L.qkv_bias)
            with sec("rope_kv"):
                q = ops.rope_and_cache(qkv, positions, self.cos_sin, kv[0], kv[1], meta.slot_mapping,
                                       self.hq, self.hkv, D, *self.kv_scales)
            with sec("attention"):
                a = ops.paged_attention(q, kv[0], kv[1], meta, cfg.attn_scale, L.sliding_window,
                                        cfg.attn_logit_softcapping, self.alibi, *self.kv_scales)
            with sec("o_gemm_rs"):
                h = self._row_parallel(a.view(a.shape[0], -1), L, "o")
            if self.is_gemma2:
                with sec("norm_ag"):
                    h = ops.rms_norm(h, L.post_attn_norm, eps, off)
                    x, residual = ops.fused_add_rms_norm(h, residual, L.pre_ff_norm, eps, off)
                with sec("down_gemm_rs"):
                    h = self._mlp(L, x)
                with sec("norm_ag"):
                    h = ops.rms_norm(h, L.post_ff_norm, eps, off)
                continue
            if mx and not cfg.is_moe:
                with sec("norm_ag"):
                    xq = ops.rms_norm_mxf8(h, L.post_attn_norm, eps, off, residual=residual)
                if L.gate_up_q.shape[0] % 256 == 0:
                    # the SiLU epilogue emits the down projection's fp8 operand directly
                    with sec("gate_up_gemm"):
                        aq = ops.linear_mxf8_silu_q(*xq, L.gate_up_q, L.gate_up_sf, act=self.act)
                    with sec("down_gemm_rs"):
                        h = self.tp.all_reduce(ops.linear_mxf8_q(*aq, L.down_q, L.down_sf))
                else:
                    with sec("gate_up_gemm"):
                        a = ops.linear_mxf8_q(*xq, L.gate_up_q, L.gate_up_sf, silu_mul=True, act=self.act)
                    with sec("down_gemm_rs"):
                        h = self._row_parallel(a, L, "down")
                continue
            with sec("norm_ag"):
                x, residual = ops.fused_add_rms_norm(h, residual, L.post_attn_norm, eps, off)
            if cfg.is_moe:
                with sec("moe"):
                    h = self._moe(L, x)
            else:
                with sec("down_gemm_rs"):
                    h = self._mlp(L, x)
        with sec("final_norm"):
            h, _ = ops.fused_add_rms_norm(h, residual, self.norm, eps, off)
        return h

    def _fused_tp_ok(self, M: int) -> bool:
        F = getattr(self.tp, "fused_tp", None)
        if F is None or self.tp.size == 1 or not F.fits(M) or self.device.type != "cuda":
            return False
        if self.is_gemma2:
            return False
        if getattr(self, "fp8", False):
            if self.act != "silu":
                return False
            # MXFP8 boundary chain (block-scaled GEMMs, quantised all-gather); fp32-scale FP8
            # checkpoints and FP8 MoE take the peer all-reduce path
            if self.cfg.is_moe or not F.mx_ok or getattr(self, "fp8_format", None) != "ue8m0":
                return False
            return all(L.gate_up_q.shape[0] % 256 == 0 for L in self.layers)
        if self.cfg.is_moe:
            # experts split over the ranks; top-k slots must fit the per-rank slot buffer
            return (self.ep_size == self.tp.size and self.cfg.num_experts_per_tok <= self.tp.size
                    and all(getattr(L, "w13_il", None) is not None for L in self.layers))
        return all(getattr(L, "gate_up_il", None) is not None for L in self.layers)

    def _forward_fused_tp(self, input_ids: torch.Tensor, positions: torch.Tensor, meta: AttentionMetadata,
                          kv_caches: List[torch.Tensor]) -> torch.Tensor:
        """Tensor-parallel forward with the collectives fused into the layer
        boundaries: the residual stream is sequence-sharded between layers;
        o_proj / down_proj reduce-scatter from their GEMM epilogues, the owner
        adds its residual, RMS-normalises and all-gathers, and QKV / gate-up
        start per tile as the gathered rows land (parallel.fused_tp).  Call
        index c of a boundary: 0 = embedding, 2l+1 = after o_proj of layer l,
        2l+2 = after down_proj of layer l.  Returns the final normalised hidden
        states (replicated)."""
        F = self.tp.fused_tp
        cfg = self.cfg
        eps, off = cfg.rms_norm_eps, cfg.norm_offset
        D = cfg.head_dim
        sec = OP_TIMER.section
        with sec("embed"):
            h = self.embed_tokens(input_ids)
        M = h.shape[0]
        # MXFP8 weights: every boundary but the last all-gathers the e4m3 operand + scales
        mx = bool(getattr(self, "fp8", False))
        with sec("norm_ag"):
            x = F.start(h, self.layers[0].input_norm, eps, off, mx=mx)
        n = len(self.layers)
        for li, L in enumerate(self.layers):
            kv = kv_caches[li]
            c_attn, c_mlp = 2 * li + 1, 2 * li + 2
            with sec("qkv_gemm"):
                if mx:
                    qkv = F.gemm_ag_mx(x, L.qkv_q, L.qkv_sf, 2 * li, L.qkv_bias)
                else:
                    qkv = F.gemm_ag(x, L.qkv, 2 * li, L.qkv_bias)
            with sec("rope_kv"):
                q = ops.rope_and_cache(qkv, positions, self.cos_sin, kv[0], kv[1], meta.slot_mapping,
                                       self.hq, self.hkv, D, *self.kv_scales)
            with sec("attention"):
                a = ops.paged_attention(q, kv[0], kv[1], meta, cfg.attn_scale, L.sliding_window,
                                        cfg.attn_logit_softcapping, self.alibi, *self.kv_scales)
            with sec("o_gemm_rs"):
                if mx:
                    F.gemm_rs_mx(*ops.quant_mxf8_act(a.view(M, -1)), L.o_q, L.o_sf, c_attn)
                else:
                    F.gemm_rs(a.view(M, -1), L.o, c_attn)
            with sec("norm_ag"):
                x = F.rs_norm_ag(M, L.post_attn_norm, eps, off, c_attn, mx=mx)
            nw = self.layers[li + 1].input_norm if li + 1 < n else self.norm
            if cfg.is_moe:
                k = cfg.num_experts_per_tok
                with sec("moe"):
                    F.moe(x, L.router, L.w13_il, L.w2, k, self.e_lo, c_attn, c_mlp)
                with sec("norm_ag"):
                    x = F.rs_norm_ag(M, nw, eps, off, c_mlp, moe_topk=k)
                continue
            if mx:
                # the gate/up epilogue emits the down projection's operand; the final norm
                # all-gathers bf16 rows for the LM head
                with sec("gate_up_gemm"):
                    aq = F.gemm_ag_mx(x, L.gate_up_q, L.gate_up_sf, c_attn, silu_q=True)
                with sec("down_gemm_rs"):
                    F.gemm_rs_mx(*aq, L.down_q, L.down_sf, c_mlp)
                with sec("norm_ag"):
                    x = F.rs_norm_ag(M, nw, eps, off, c_mlp, mx=li + 1 < n)
                continue
            with sec("gate_up_gemm"):
                act = F.gemm_ag(x, L.gate_up_il, c_attn, silu_mul=True, act=self.act)
            with sec("down_gemm_rs"):
                F.gemm_rs(act, L.down, c_mlp)
            with sec("norm_ag"):
                x = F.rs_norm_ag(M, nw, eps, off, c_mlp)
        # the LM head reads every owner's final rows from the local gather buffer
        with sec("final_norm"):
            F.wait_gathered(M, 2 * n)
            F.end_step()
        return x

    def compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        """h [n, H] -> logits [n, vocab] (gathered over TP ranks): bf16 on the GPU (fp32
        with a final softcap), fp32 on the CPU."""
        with OP_TIMER.section("lm_head"):
            return self._compute_logits(h)

    def _compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        if getattr(self, "lm_head_q", None) is not None:
            logits = ops.linear_fp8(h, self.lm_head_q, self.lm_head_s, wsf=getattr(self, "lm_head_sf", None))
        else:
            logits = ops.linear(h, self.lm_head_weight)
        if self.tp.size > 1:
            logits = self.tp.all_gather_last_dim(logits)
        logits = logits[:, : self.cfg.vocab_size]
        cap = self.cfg.final_logit_softcapping
        if cap:
            logits = cap * torch.tanh(logits.float() / cap)
        elif not logits.is_cuda:
            logits = logits.float()
        # on the GPU the logits stay in the GEMM's bf16 (a strided view past a padded
        # vocabulary): the sampling kernel reads bf16 rows directly, host-side paths cast
        return logits


def _pad_vocab(v: int, tps: int) -> int:
    return (v + tps - 1) // tps * tps


def moe_forward_local(L, h: torch.Tensor, cfg: ModelConfig, e_lo: int, e_hi: int, tp) -> torch.Tensor:
    """Top-k softmax routed MoE with this rank's experts [e_lo, e_hi); the
    partial sums are reduced over the group by the caller's all-reduce.  This
    is the dense-loop oracle; the GPU path replaces it with the grouped-GEMM
    kernels in `rusteeze_b200.parallel.moe`."""
    logits = ops.linear(h, L.router).float()
    w, idx = ref.moe_topk_softmax(logits, cfg.num_experts_per_tok)
    out = torch.zeros(h.shape[0], h.shape[1], dtype=torch.float32, device=h.device)
    for e in range(e_lo, e_hi):
        rows, slot = (idx == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        xe = h.index_select(0, rows)
        gu = ops.linear(xe, L.w13[e - e_lo])
        y = ops.linear(ops.silu_mul(gu), L.w2[e - e_lo])
        out.index_add_(0, rows, y.float() * w[rows, slot].unsqueeze(1))
    out = out.to(h.dtype)
    return tp.all_reduce(out) if (tp.size > 1) else out
