"""FP8 block-scaled weight quantisation at load time.

Every projection weight W [N, K] becomes e4m3 Wq plus fp32 scales S
[ceil(N/128), K/128], one per 128x128 block (amax / 448), the DeepSeek-style
block format named by the Llama-3-8B FP8 serving configuration.  The
reference's quantizers (crates/rusteeze-engine/src/quantization.rs:238-531,
crates/rusteeze-tensor/src/quantize.rs:147-476) are CPU-side and dequantise
before each matmul; here the GPU GEMM consumes Wq directly (gemm_fp8.cu)
and activations are quantised 1x128 on the fly.

gate/up is quantised in its 64-row interleaved layout so the fp8 GEMM's
SiLU(gate)*up epilogue applies, exactly as for bf16.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref


def _q(w: torch.Tensor):
    q, s = ref.quant_fp8_weight(w)
    return nn.Parameter(q, requires_grad=False), nn.Parameter(s.contiguous(), requires_grad=False)


def _drop(owner, name: str) -> None:
    p = getattr(owner, name)
    setattr(owner, name, nn.Parameter(torch.empty(0, dtype=p.dtype, device=p.device), requires_grad=False))


@torch.no_grad()
def quantize_model_fp8(model) -> None:
    """Replaces the bf16 projection weights of a DecoderLM by e4m3 + scales (in place)."""
    if model.cfg.is_moe:
        raise NotImplementedError("fp8 quantisation of MoE experts is not supported")
    for L in model.layers:
        L.qkv_q, L.qkv_s = _q(L.qkv)
        _drop(L, "qkv")
        L.o_q, L.o_s = _q(L.o)
        _drop(L, "o")
        gu = L.gate_up_il if getattr(L, "gate_up_il", None) is not None else ops.interleave_gate_up(L.gate_up)
        L.gate_up_q, L.gate_up_s = _q(gu)
        L.gate_up_il = None
        _drop(L, "gate_up")
        L.down_q, L.down_s = _q(L.down)
        _drop(L, "down")
    if model.lm_head is not None and model.lm_head.shape[0] % 128 == 0:
        model.lm_head_q, model.lm_head_s = _q(model.lm_head)
        _drop(model, "lm_head")
    model.fp8 = True
    if model.device.type == "cuda":
        torch.cuda.empty_cache()
