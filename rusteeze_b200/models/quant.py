"""FP8 block-scaled weight quantisation at load time.

Every projection weight W [N, K] becomes e4m3 Wq plus one scale per 128x128
block, the DeepSeek-style block format named by the Llama-3-8B FP8 serving
configuration.  The reference's quantizers (crates/rusteeze-engine/src/
quantization.rs:238-531, crates/rusteeze-tensor/src/quantize.rs:147-476) are
CPU-side and dequantise before each matmul; here the GPU GEMM consumes Wq
directly and activations are quantised 1x128 on the fly.

Two scale formats:
  "ue8m0" (default)  power-of-two scales (the smallest 2^e with amax/2^e <=
                     448), stored as fp32 `<name>_s` plus the GEMM's packed
                     exponent chunks `<name>_sf`; the sm_100a block-scaled MMA
                     (kind::mxf8f6f4) applies them in the tensor core;
  "fp32"             arbitrary fp32 scales amax/448 (`<name>_s`), applied per
                     128-K block in the GEMM epilogue (gemm_fp8.cu) -- the
                     format of checkpoints quantised elsewhere.

gate/up is quantised in its 64-row interleaved layout so the fp8 GEMM's
SiLU(gate)*up epilogue applies, exactly as for bf16.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref


def _param(t: torch.Tensor) -> nn.Parameter:
    return nn.Parameter(t.contiguous(), requires_grad=False)


def _quantize(owner, name: str, w: torch.Tensor, fmt: str) -> None:
    if fmt == "ue8m0":
        q, s = ref.quant_mxf8_weight(w)
        setattr(owner, name + "_sf", _param(ref.pack_block_scales_ue8m0(s)))
    elif fmt == "fp32":
        q, s = ref.quant_fp8_weight(w)
    else:
        raise ValueError(f"unknown fp8 scale format {fmt!r}")
    setattr(owner, name + "_q", _param(q))
    setattr(owner, name + "_s", _param(s))


def _drop(owner, name: str) -> None:
    p = getattr(owner, name)
    setattr(owner, name, nn.Parameter(torch.empty(0, dtype=p.dtype, device=p.device), requires_grad=False))


@torch.no_grad()
def quantize_model_fp8(model, scale_format: str = "ue8m0") -> None:
    """Replaces the bf16 projection weights of a DecoderLM by e4m3 + scales (in place)."""
    if model.cfg.is_moe:
        raise NotImplementedError("fp8 quantisation of MoE experts is not supported")
    for L in model.layers:
        _quantize(L, "qkv", L.qkv, scale_format)
        _drop(L, "qkv")
        _quantize(L, "o", L.o, scale_format)
        _drop(L, "o")
        gu = L.gate_up_il if getattr(L, "gate_up_il", None) is not None else ops.interleave_gate_up(L.gate_up)
        _quantize(L, "gate_up", gu, scale_format)
        L.gate_up_il = None
        _drop(L, "gate_up")
        _quantize(L, "down", L.down, scale_format)
        _drop(L, "down")
    if model.lm_head is not None and model.lm_head.shape[0] % 128 == 0:
        _quantize(model, "lm_head", model.lm_head, scale_format)
        _drop(model, "lm_head")
    model.fp8 = True
    model.fp8_format = scale_format
    if model.device.type == "cuda":
        torch.cuda.empty_cache()
