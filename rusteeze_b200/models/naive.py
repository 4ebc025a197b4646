"""Naive full-recompute forward: the end-to-end oracle.

Computes logits for every position of ONE sequence from scratch with dense
causal attention (no KV cache, no paging, no batching), the way the
reference's eager candle forward does (crates/rusteeze-model/src/
architectures/llama.rs:278-339 with common.rs:234-317 attention and
common.rs:354-361 MLP).  The paged, continuously batched engine must
reproduce its greedy tokens exactly.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from rusteeze_b200.models.decoder import DecoderLM
from rusteeze_b200.ops import reference as ref


@torch.no_grad()
def naive_logits(model: DecoderLM, ids, observer=None) -> torch.Tensor:
    """`observer(name, x)`, when given, sees the input of every attention / MLP linear under
    its HF name (calibration for integer quantization), and the final normalised hidden
    states as "lm_head" (the embedding oracle)."""
    cfg = model.cfg
    obs = observer or (lambda name, x: None)
    assert model.tp.size == 1
    ids = torch.as_tensor(ids, dtype=torch.long)
    n = ids.numel()
    D, hq, hkv = cfg.head_dim, model.hq, model.hkv
    eps, off = cfg.rms_norm_eps, cfg.norm_offset
    f = lambda t: t.float()  # noqa: E731
    h = f(model.embed)[ids] * cfg.embed_scale
    pos = torch.arange(n)
    cs = model.cos_sin.float().cpu()
    for li, L in enumerate(model.layers):
        x = ref.rms_norm(h, f(L.input_norm), eps, off)
        pre = f"model.layers.{li}."
        for nm in ("q_proj", "k_proj", "v_proj"):
            obs(pre + "self_attn." + nm, x)
        qkv = x @ f(L.qkv).t()
        if L.qkv_bias is not None:
            qkv = qkv + f(L.qkv_bias)
        q = qkv[:, :hq * D].view(n, hq, D).clone()
        k = qkv[:, hq * D:(hq + hkv) * D].view(n, hkv, D).clone()
        v = qkv[:, (hq + hkv) * D:].view(n, hkv, D)
        ref.rope(q, k, pos, cs)
        kk = k.repeat_interleave(hq // hkv, 1)
        vv = v.repeat_interleave(hq // hkv, 1)
        s = torch.einsum("qhd,khd->hqk", q, kk) * cfg.attn_scale
        if cfg.attn_logit_softcapping:
            c = cfg.attn_logit_softcapping
            s = c * torch.tanh(s / c)
        if model.alibi is not None:
            s = s + ref.alibi_bias(model.alibi.float().cpu(), pos, pos)
        mask = torch.ones(n, n, dtype=torch.bool).triu(1)
        w = L.sliding_window
        if w:
            mask |= torch.ones(n, n, dtype=torch.bool).tril(-w)
        s = s.masked_fill(mask, float("-inf"))
        a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv).reshape(n, hq * D)
        obs(pre + "self_attn.o_proj", a)
        o = a @ f(L.o).t()
        if model.is_gemma2:
            o = ref.rms_norm(o, f(L.post_attn_norm), eps, off)
            h = h + o
            x = ref.rms_norm(h, f(L.pre_ff_norm), eps, off)
        else:
            h = h + o
            x = ref.rms_norm(h, f(L.post_attn_norm), eps, off)
        if cfg.is_moe:
            logits = x @ f(L.router).t()
            wts, idx = ref.moe_topk_softmax(logits, cfg.num_experts_per_tok)
            y = torch.zeros_like(x)
            for t in range(n):
                for j in range(cfg.num_experts_per_tok):
                    e = int(idx[t, j])
                    gu = x[t] @ f(L.w13[e]).t()
                    g, u = gu.chunk(2)
                    y[t] += wts[t, j] * ((F.silu(g) * u) @ f(L.w2[e]).t())
        else:
            obs(pre + "mlp.gate_proj", x)
            obs(pre + "mlp.up_proj", x)
            gu = x @ f(L.gate_up).t()
            g, u = gu.chunk(2, dim=-1)
            act = F.gelu(g, approximate="tanh") if model.act == "gelu_tanh" else F.silu(g)
            obs(pre + "mlp.down_proj", act * u)
            y = (act * u) @ f(L.down).t()
        if model.is_gemma2:
            y = ref.rms_norm(y, f(L.post_ff_norm), eps, off)
        h = h + y
    h = ref.rms_norm(h, f(model.norm), eps, off)
    obs("lm_head", h)
    logits = h @ f(model.lm_head_weight).t()
    logits = logits[:, :cfg.vocab_size]
    if cfg.final_logit_softcapping:
        c = cfg.final_logit_softcapping
        logits = c * torch.tanh(logits / c)
    return logits


@torch.no_grad()
def naive_greedy(model: DecoderLM, prompt, max_new: int):
    ids = list(prompt)
    for _ in range(max_new):
        ids.append(int(naive_logits(model, ids)[-1].argmax()))
    return ids[len(prompt):]
