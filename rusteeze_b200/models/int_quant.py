"""Integer weight quantization: the codecs, the offline algorithms, and the GPTQ / AWQ / INT8
checkpoint formats.

Covers what the reference's quantization library does (crates/rusteeze-tensor/src/
quantize.rs:11-146 `QuantMethod` / `QuantConfig` / `QuantState`, :147-328 int8 and grouped
quantize / dequantize, `QuantizedLinear`, int4 packing, :333-401 GPTQ / AWQ states and
`QuantStats`; crates/rusteeze-engine/src/quantization.rs:21-603 `QuantEngine` with GPTQ,
AWQ, SmoothQuant and a calibration collector), written from the published methods:

* GPTQ -- Frantar et al., "GPTQ: Accurate Post-Training Quantization for Generative
  Pre-trained Transformers", 2022: columns quantized in order with the remaining columns
  corrected through the inverse-Hessian Cholesky factor of the layer inputs (the
  reference's `quantize_gptq` carries a scalar error term instead).
* AWQ -- Lin et al., "AWQ: Activation-aware Weight Quantization", 2023: per-input-channel
  scales s = mean|x|^a with a searched on a grid, the weights quantized as W diag(s).
* SmoothQuant -- Xiao et al., 2022: s_j = max|x_j|^a / max|W_j|^(1-a) moves activation
  outliers into the weights.

Serving: the engine's tensor-core formats are bf16 and block-scaled FP8 (MXFP8).  Integer
checkpoints are dequantized when they are loaded (`dequantize_checkpoint_tensor`, used by
`models.loader`), so they run on the bf16 kernels, or on the FP8 ones with
`quantization.method: fp8_block`.  There is no integer GEMM kernel.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Tuple

import torch

# ----------------------------------------------------------------------------- config
METHODS = ("none", "int8", "int4", "fp8_e4m3", "fp8_e5m2", "gptq", "awq", "smoothquant")


@dataclass
class QuantConfig:
    """Quantization settings (the reference's `QuantConfig`): `bits` per weight, scales per
    `group_size` input columns (0 or per_channel: one per output row), symmetric or with a
    zero point, and layer names left in full precision."""
    method: str = "none"
    bits: int = 16
    group_size: int = 128
    per_channel: bool = True
    symmetric: bool = True
    exclude_layers: List[str] = field(default_factory=list)
    damp_percent: float = 0.01          # GPTQ: Hessian damping, as a fraction of its mean diagonal
    act_order: bool = False             # GPTQ: columns by decreasing Hessian diagonal
    smooth_alpha: float = 0.5           # SmoothQuant migration strength

    def __post_init__(self) -> None:
        if self.method not in METHODS:
            raise ValueError(f"unknown quantization method {self.method!r}; known: {METHODS}")

    @classmethod
    def int8(cls) -> "QuantConfig":
        return cls(method="int8", bits=8, group_size=0)

    @classmethod
    def int4(cls, group_size: int = 128) -> "QuantConfig":
        return cls(method="int4", bits=4, group_size=group_size, symmetric=False)

    @classmethod
    def fp8(cls) -> "QuantConfig":
        return cls(method="fp8_e4m3", bits=8)

    @classmethod
    def gptq(cls, bits: int = 4, group_size: int = 128) -> "QuantConfig":
        return cls(method="gptq", bits=bits, group_size=group_size, symmetric=False)

    @classmethod
    def awq(cls, bits: int = 4, group_size: int = 128) -> "QuantConfig":
        return cls(method="awq", bits=bits, group_size=group_size, symmetric=False)

    def exclude(self, layers: Iterable[str]) -> "QuantConfig":
        self.exclude_layers = list(layers)
        return self

    def with_group_size(self, group_size: int) -> "QuantConfig":
        self.group_size = group_size
        return self

    def skips(self, name: str) -> bool:
        return any(x and x in name for x in self.exclude_layers)


@dataclass
class QuantState:
    """Dequantization data: w = scale * (q - zero), scales / zeros per (row, group)."""
    scales: torch.Tensor
    zero_points: Optional[torch.Tensor]
    group_size: int
    original_shape: Tuple[int, ...]
    original_dtype: torch.dtype
    bits: int = 8


@dataclass
class QuantStats:
    layers_quantized: int = 0
    original_size: int = 0
    quantized_size: int = 0
    mean_error: float = 0.0
    max_error: float = 0.0

    def compression_ratio(self) -> float:
        return self.original_size / self.quantized_size if self.quantized_size else 0.0

    def add(self, w: torch.Tensor, w_hat: torch.Tensor, qbytes: int) -> None:
        err = (w.float() - w_hat.float()).abs()
        n = self.layers_quantized
        self.mean_error = (self.mean_error * n + float(err.mean())) / (n + 1)
        self.max_error = max(self.max_error, float(err.max()))
        self.layers_quantized = n + 1
        self.original_size += w.numel() * w.element_size()
        self.quantized_size += qbytes


# ----------------------------------------------------------------------------- codecs
def _qrange(bits: int, symmetric: bool) -> Tuple[int, int]:
    if symmetric:
        m = (1 << (bits - 1)) - 1
        return -m, m
    return 0, (1 << bits) - 1


def _scale_zero(lo: torch.Tensor, hi: torch.Tensor, bits: int, symmetric: bool):
    """Scale and zero point covering [lo, hi] (per row or group)."""
    qmin, qmax = _qrange(bits, symmetric)
    if symmetric:
        amax = torch.maximum(lo.abs(), hi.abs()).clamp_min(1e-12)
        return amax / qmax, None
    lo = torch.minimum(lo, torch.zeros_like(lo))
    hi = torch.maximum(hi, torch.zeros_like(hi))
    scale = ((hi - lo) / (qmax - qmin)).clamp_min(1e-12)
    zero = torch.round(-lo / scale).clamp(qmin, qmax)
    return scale, zero


def _quant(w: torch.Tensor, scale: torch.Tensor, zero: Optional[torch.Tensor], bits: int, symmetric: bool):
    qmin, qmax = _qrange(bits, symmetric)
    q = torch.round(w / scale) + (zero if zero is not None else 0)
    return q.clamp(qmin, qmax)


def _dequant(q: torch.Tensor, scale: torch.Tensor, zero: Optional[torch.Tensor]) -> torch.Tensor:
    return (q.float() - (zero if zero is not None else 0)) * scale


def quantize_int8(w: torch.Tensor, per_channel: bool = True, symmetric: bool = True):
    """int8 codes (uint8 when asymmetric) with one scale per row or per tensor."""
    x = w.float()
    if per_channel:
        lo, hi = x.amin(dim=-1, keepdim=True), x.amax(dim=-1, keepdim=True)
    else:
        lo, hi = x.min().reshape(1, 1), x.max().reshape(1, 1)
    scale, zero = _scale_zero(lo, hi, 8, symmetric)
    q = _quant(x, scale, zero, 8, symmetric).to(torch.int8 if symmetric else torch.uint8)
    return q, QuantState(scale, zero, 0, tuple(w.shape), w.dtype, 8)


def dequantize_int8(q: torch.Tensor, state: QuantState) -> torch.Tensor:
    return _dequant(q, state.scales, state.zero_points).to(state.original_dtype)


def quantize_grouped(w: torch.Tensor, bits: int = 4, group_size: int = 128, symmetric: bool = False):
    """Codes [N, K] (uint8 holding 0..2^bits-1 when asymmetric, int8 when symmetric) with a
    scale (and zero) per row and per `group_size` columns; K must divide by group_size."""
    N, K = w.shape
    g = group_size if group_size > 0 else K
    if K % g:
        raise ValueError(f"{K} columns do not divide into groups of {g}")
    x = w.float().view(N, K // g, g)
    scale, zero = _scale_zero(x.amin(-1, keepdim=True), x.amax(-1, keepdim=True), bits, symmetric)
    q = _quant(x, scale, zero, bits, symmetric).view(N, K)
    q = q.to(torch.int8 if symmetric else torch.uint8)
    return q, QuantState(scale.view(N, K // g), None if zero is None else zero.view(N, K // g), g,
                         (N, K), w.dtype, bits)


def dequantize_grouped(q: torch.Tensor, state: QuantState) -> torch.Tensor:
    N, K = state.original_shape
    g = state.group_size
    z = None if state.zero_points is None else state.zero_points.view(N, K // g, 1)
    return _dequant(q.view(N, K // g, g), state.scales.view(N, K // g, 1), z).view(N, K).to(state.original_dtype)


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """Two 4-bit codes (0..15) per byte along the last dimension, the even one in the low
    nibble."""
    c = codes.to(torch.uint8)
    if c.shape[-1] % 2:
        raise ValueError("int4 packing needs an even last dimension")
    return (c[..., 0::2] & 0xF) | ((c[..., 1::2] & 0xF) << 4)


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    p = packed.to(torch.uint8)
    out = torch.empty(*p.shape[:-1], p.shape[-1] * 2, dtype=torch.uint8, device=p.device)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


class QuantizedLinear:
    """Weight-only quantized linear layer (the reference's `QuantizedLinear`): integer codes
    and scales are kept, `forward` dequantizes and multiplies (a reference path, not a
    serving kernel)."""

    def __init__(self, q: torch.Tensor, state: QuantState, bias: Optional[torch.Tensor] = None):
        self.q, self.state, self.bias = q, state, bias

    @classmethod
    def from_float(cls, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
                   cfg: Optional[QuantConfig] = None) -> "QuantizedLinear":
        cfg = cfg or QuantConfig.int8()
        if cfg.bits == 8 and cfg.group_size == 0:
            q, st = quantize_int8(w, cfg.per_channel, cfg.symmetric)
        else:
            q, st = quantize_grouped(w, cfg.bits, cfg.group_size, cfg.symmetric)
            if cfg.bits == 4:
                q = pack_int4(q.to(torch.int16).add(8).to(torch.uint8) if cfg.symmetric else q)
        return cls(q, st, bias)

    def weight(self) -> torch.Tensor:
        st = self.state
        if st.bits == 4:
            codes = unpack_int4(self.q)
            if st.zero_points is None:
                codes = codes.to(torch.int16) - 8
            return dequantize_grouped(codes, st)
        if st.group_size:
            return dequantize_grouped(self.q, st)
        return dequantize_int8(self.q, st)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = x.float() @ self.weight().float().t()
        if self.bias is not None:
            y = y + self.bias.float()
        return y.to(x.dtype)

    __call__ = forward

    def memory_savings(self) -> float:
        full = math.prod(self.state.original_shape) * 2          # vs bf16
        qb = self.q.numel() * self.q.element_size() + self.state.scales.numel() * 4
        if self.state.zero_points is not None:
            qb += self.state.zero_points.numel() * 4
        return 1.0 - qb / full


# ----------------------------------------------------------------------------- calibration
class CalibrationCollector:
    """Per-layer input statistics from calibration forwards (the reference's
    `CalibrationCollector` / `LayerStats`): per-input-channel max |x| and mean |x|, the
    sample count, and (when `keep_inputs`) up to `max_rows` input rows for GPTQ / AWQ."""

    def __init__(self, keep_inputs: bool = False, max_rows: int = 4096):
        self.keep_inputs, self.max_rows = keep_inputs, max_rows
        self.absmax: Dict[str, torch.Tensor] = {}
        self.abssum: Dict[str, torch.Tensor] = {}
        self.count: Dict[str, int] = {}
        self.inputs: Dict[str, List[torch.Tensor]] = {}

    def record(self, name: str, x: torch.Tensor) -> None:
        x = x.detach().float().reshape(-1, x.shape[-1]).cpu()
        a = x.abs()
        if name in self.absmax:
            self.absmax[name] = torch.maximum(self.absmax[name], a.amax(0))
            self.abssum[name] += a.sum(0)
            self.count[name] += x.shape[0]
        else:
            self.absmax[name], self.abssum[name], self.count[name] = a.amax(0), a.sum(0), x.shape[0]
        if self.keep_inputs:
            rows = self.inputs.setdefault(name, [])
            have = sum(r.shape[0] for r in rows)
            if have < self.max_rows:
                rows.append(x[: self.max_rows - have])

    def get_stats(self, name: str) -> Optional[Dict[str, torch.Tensor]]:
        if name not in self.count:
            return None
        return {"absmax": self.absmax[name], "absmean": self.abssum[name] / self.count[name],
                "count": torch.tensor(self.count[name])}

    def layer_inputs(self, name: str) -> torch.Tensor:
        return torch.cat(self.inputs[name], 0)

    def names(self) -> List[str]:
        return list(self.count)


def hessian(x: torch.Tensor) -> torch.Tensor:
    """H = 2/T X^T X of the layer inputs X [T, K] (the GPTQ objective's Hessian)."""
    x = x.double().reshape(-1, x.shape[-1])
    return (2.0 / max(1, x.shape[0])) * (x.t() @ x)


# ----------------------------------------------------------------------------- GPTQ
@torch.no_grad()
def gptq_quantize(w: torch.Tensor, H: torch.Tensor, bits: int = 4, group_size: int = 128,
                  damp_percent: float = 0.01, act_order: bool = False, symmetric: bool = False,
                  block: int = 128):
    """GPTQ on one layer, w [N, K], H [K, K].  Returns (codes [N, K] in the original column
    order, scales [N, G], zeros [N, G] or None, g_idx [K] = group of each column), with
    w_hat[:, k] = scales[:, g_idx[k]] * (codes[:, k] - zeros[:, g_idx[k]]).

    Following the paper: dead inputs (zero Hessian diagonal) get weight 0; H is damped by
    damp_percent of its mean diagonal; U = upper Cholesky factor of H^-1; columns are taken
    in order (or by decreasing diagonal with act_order) in blocks, each column quantized
    with its group's scale (computed when the group starts, from the updated weights), its
    error divided by U[i, i] and propagated into the later columns of the block by row i of
    U, and the block's errors into the columns after it."""
    W = w.double().clone()
    N, K = W.shape
    H = H.double().clone()
    g = group_size if group_size > 0 else K
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    perm = torch.argsort(torch.diag(H), descending=True) if act_order else torch.arange(K)
    W, H = W[:, perm], H[perm][:, perm]
    damp = damp_percent * torch.mean(torch.diag(H))
    H += damp * torch.eye(K, dtype=H.dtype)
    L = torch.linalg.cholesky(H)
    U = torch.linalg.cholesky(torch.cholesky_inverse(L), upper=True)
    Q = torch.zeros_like(W)
    G = (K + g - 1) // g
    scales = torch.zeros(N, G, dtype=torch.float64)
    zeros = None if symmetric else torch.zeros(N, G, dtype=torch.float64)
    # groups follow the ORIGINAL column index (g_idx), so with act_order a group's scale is
    # set by the first of its columns in processing order
    group_of = perm // g
    seen = torch.zeros(G, dtype=torch.bool)
    for b0 in range(0, K, block):
        b1 = min(K, b0 + block)
        W1 = W[:, b0:b1].clone()
        E1 = torch.zeros_like(W1)
        U1 = U[b0:b1, b0:b1]
        for i in range(b1 - b0):
            col = b0 + i
            gi = int(group_of[col])
            if not bool(seen[gi]):
                # columns of this group in processing order: the current one and later ones
                members = (group_of[col:] == gi).nonzero().flatten() + col
                cur = torch.cat([W1[:, members[members < b1] - b0], W[:, members[members >= b1]]], 1)
                s, z = _scale_zero(cur.amin(1), cur.amax(1), bits, symmetric)
                scales[:, gi] = s
                if zeros is not None:
                    zeros[:, gi] = z
                seen[gi] = True
            s = scales[:, gi]
            z = None if zeros is None else zeros[:, gi]
            wcol = W1[:, i]
            qcol = _quant(wcol, s, z, bits, symmetric)
            dq = _dequant(qcol, s, z)
            Q[:, col] = qcol
            err = (wcol - dq) / U1[i, i]
            W1[:, i:] -= err.unsqueeze(1) * U1[i, i:].unsqueeze(0)
            E1[:, i] = err
        W[:, b1:] -= E1 @ U[b0:b1, b1:]
    inv = torch.argsort(perm)
    codes = Q[:, inv]
    g_idx = (torch.arange(K) // g).to(torch.int32)
    dtype = torch.int8 if symmetric else torch.uint8
    return (codes.to(dtype), scales.float(), None if zeros is None else zeros.float(), g_idx)


def dequantize_gptq(codes: torch.Tensor, scales: torch.Tensor, zeros: Optional[torch.Tensor],
                    g_idx: torch.Tensor) -> torch.Tensor:
    gi = g_idx.long()
    s = scales[:, gi]
    z = 0 if zeros is None else zeros[:, gi]
    return (codes.float() - z) * s


# ----------------------------------------------------------------------------- AWQ
@torch.no_grad()
def awq_search_scales(w: torch.Tensor, x: torch.Tensor, bits: int = 4, group_size: int = 128,
                      grid: int = 20) -> Tuple[torch.Tensor, float]:
    """Per-input-channel scales s = mean|x|^a (normalised so max * min = 1) with a in
    {0, 1/grid, ..., (grid-1)/grid} chosen to minimise ||x W^T - x (Q(W diag s) / s)^T||^2.
    Returns (s [K], the chosen a); a = 0 gives s = 1 (plain grouped quantization)."""
    W = w.float()
    X = x.float().reshape(-1, x.shape[-1])
    ref = X @ W.t()
    xm = X.abs().mean(0).clamp_min(1e-8)
    best, best_s, best_a = float("inf"), torch.ones_like(xm), 0.0
    for i in range(grid):
        a = i / grid
        s = xm.pow(a)
        s = s / (s.max() * s.min()).sqrt()
        q, st = quantize_grouped(W * s, bits, group_size, symmetric=False)
        w_hat = dequantize_grouped(q, st).float() / s
        loss = float(((X @ w_hat.t()) - ref).pow(2).mean())
        if loss < best:
            best, best_s, best_a = loss, s, a
    return best_s, best_a


@torch.no_grad()
def awq_quantize(w: torch.Tensor, x: torch.Tensor, bits: int = 4, group_size: int = 128, grid: int = 20):
    """AWQ on one layer: (codes [N, K] of W diag(s), QuantState, s [K]).  The serving form
    multiplies the layer's input by 1/s, which `fold_input_scale` moves into the weight
    (or norm) that produces that input."""
    s, _ = awq_search_scales(w, x, bits, group_size, grid)
    q, st = quantize_grouped(w.float() * s, bits, group_size, symmetric=False)
    return q, st, s


def fold_input_scale(producer: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """Divides the producer of a layer's input by s: a norm weight [K] or the output rows of
    the previous linear [K, *]."""
    return producer.float() / (s if producer.dim() == 1 else s.unsqueeze(1))


# ----------------------------------------------------------------------------- SmoothQuant
def smoothquant_scales(act_absmax: torch.Tensor, weights: Iterable[torch.Tensor], alpha: float = 0.5) -> torch.Tensor:
    """s_j = max|x_j|^alpha / max|W_:,j|^(1-alpha) over the linears that read the same input."""
    wmax = torch.stack([w.float().abs().amax(0) for w in weights]).amax(0)
    s = act_absmax.float().clamp_min(1e-5).pow(alpha) / wmax.clamp_min(1e-5).pow(1 - alpha)
    return s.clamp_min(1e-5)


def apply_smoothing(norm_weight: torch.Tensor, linears: List[torch.Tensor], s: torch.Tensor):
    """x -> x / s (folded into the norm), W -> W diag(s): the product is unchanged."""
    return norm_weight.float() / s, [w.float() * s for w in linears]


# ----------------------------------------------------------------------------- checkpoint formats
# GPTQ layout (AutoGPTQ convention, `quant_method: gptq`):
#   qweight int32 [K * bits / 32, N]: 32/bits consecutive input columns per word, lowest first
#   qzeros  int32 [G, N * bits / 32]: zero points packed along the outputs, stored minus one
#           (`checkpoint_format: gptq`; `gptq_v2` stores them as they are)
#   scales  fp16  [G, N];  g_idx int32 [K]: group of each input column
# AWQ layout (AutoAWQ "gemm" convention, `quant_method: awq`):
#   qweight int32 [K, N * bits / 32]: 32/bits outputs per word in the interleaved order
#           0 2 4 6 1 3 5 7 (4-bit);  qzeros int32 [G, N * bits / 32] packed the same way
#   scales  fp16  [G, N]
# INT8 weight-only (`weight` int8 [N, K] with `weight_scale` [N] or [N, 1]).
_AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def _pack_words(codes: torch.Tensor, bits: int, dim: int, order=None) -> torch.Tensor:
    """Packs unsigned codes along `dim` into int32 words (32/bits codes per word, code i of
    a word at bit bits * i; `order[i]` names the element stored in slot i)."""
    per = 32 // bits
    c = codes.to(torch.int64).movedim(dim, -1)
    if c.shape[-1] % per:
        raise ValueError(f"dimension {c.shape[-1]} is not a multiple of {per}")
    c = c.reshape(*c.shape[:-1], c.shape[-1] // per, per)
    if order is not None:
        c = c[..., list(order)]
    w = torch.zeros(c.shape[:-1], dtype=torch.int64)
    for i in range(per):
        w |= (c[..., i] & ((1 << bits) - 1)) << (bits * i)
    w = torch.where(w >= 2 ** 31, w - 2 ** 32, w)
    return w.to(torch.int32).movedim(-1, dim).contiguous()


def _unpack_words(words: torch.Tensor, bits: int, dim: int, order=None) -> torch.Tensor:
    per = 32 // bits
    w = words.to(torch.int64).movedim(dim, -1) & 0xFFFFFFFF
    c = torch.stack([(w >> (bits * i)) & ((1 << bits) - 1) for i in range(per)], -1)
    if order is not None:
        inv = [0] * per
        for slot, elem in enumerate(order):
            inv[elem] = slot
        c = c[..., inv]
    c = c.reshape(*c.shape[:-2], c.shape[-2] * per)
    return c.movedim(-1, dim)


def pack_gptq(codes: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, g_idx: torch.Tensor,
              bits: int = 4, v2: bool = False) -> Dict[str, torch.Tensor]:
    """codes [N, K] (0..2^bits-1), scales / zeros [N, G] -> the GPTQ tensors of one layer."""
    z = zeros.round().to(torch.int64) - (0 if v2 else 1)
    return {"qweight": _pack_words(codes.t().contiguous(), bits, 0),
            "qzeros": _pack_words(z.t().contiguous() & ((1 << bits) - 1), bits, 1),
            "scales": scales.t().contiguous().to(torch.float16),
            "g_idx": g_idx.to(torch.int32)}


def unpack_gptq(t: Dict[str, torch.Tensor], bits: int = 4, v2: bool = False) -> torch.Tensor:
    """The GPTQ tensors of one layer -> dequantized weight [N, K] (fp32)."""
    codes = _unpack_words(t["qweight"], bits, 0)                      # [K, N]
    zeros = _unpack_words(t["qzeros"], bits, 1) + (0 if v2 else 1)     # [G, N]
    scales = t["scales"].float()                                      # [G, N]
    K = codes.shape[0]
    g_idx = t.get("g_idx")
    if g_idx is None:
        g_idx = torch.arange(K) // (K // scales.shape[0])
    gi = g_idx.long()
    return ((codes.float() - zeros[gi].float()) * scales[gi]).t().contiguous()


def pack_awq(codes: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, bits: int = 4) -> Dict[str, torch.Tensor]:
    """codes [N, K] (0..2^bits-1), scales / zeros [N, G] -> the AWQ tensors of one layer."""
    return {"qweight": _pack_words(codes.t().contiguous(), bits, 1, _AWQ_ORDER),
            "qzeros": _pack_words(zeros.round().t().contiguous(), bits, 1, _AWQ_ORDER),
            "scales": scales.t().contiguous().to(torch.float16)}


def unpack_awq(t: Dict[str, torch.Tensor], bits: int = 4) -> torch.Tensor:
    codes = _unpack_words(t["qweight"], bits, 1, _AWQ_ORDER)          # [K, N]
    zeros = _unpack_words(t["qzeros"], bits, 1, _AWQ_ORDER)           # [G, N]
    scales = t["scales"].float()
    K = codes.shape[0]
    gi = torch.arange(K) // (K // scales.shape[0])
    return ((codes.float() - zeros[gi].float()) * scales[gi]).t().contiguous()


def checkpoint_quant_config(hf_config: Dict) -> Optional[Dict]:
    """The `quantization_config` of an HF config.json when it names an integer format this
    loader reads (gptq, awq, int8 weight-only); None otherwise."""
    qc = hf_config.get("quantization_config") or None
    if not qc:
        return None
    m = str(qc.get("quant_method", "")).lower()
    if m in ("gptq", "awq", "int8"):
        return dict(qc, quant_method=m)
    return None


def dequantize_checkpoint_tensor(get: Callable[[str], torch.Tensor], has: Callable[[str], bool],
                                 prefix: str, qc: Dict) -> Optional[torch.Tensor]:
    """Weight [N, K] of layer `prefix` (e.g. "model.layers.0.mlp.down_proj") from its
    integer tensors, or None when the layer is stored in full precision."""
    m = qc["quant_method"]
    bits = int(qc.get("bits", 8 if m == "int8" else 4))
    if m in ("gptq", "awq") and has(prefix + ".qweight"):
        t = {k: get(prefix + "." + k) for k in ("qweight", "qzeros", "scales", "g_idx") if has(prefix + "." + k)}
        if m == "gptq":
            return unpack_gptq(t, bits, v2=str(qc.get("checkpoint_format", "gptq")) == "gptq_v2")
        w = unpack_awq(t, bits)
        # AWQ checkpoints fold 1/s into the layer that produces the input; one written with
        # the producer left as it is carries s (input_scale) and is divided here
        if has(prefix + ".input_scale"):
            w = w / get(prefix + ".input_scale").float()
        return w
    if has(prefix + ".weight_scale"):
        w = get(prefix + ".weight")
        if w.dtype in (torch.int8, torch.uint8):
            s = get(prefix + ".weight_scale").float().reshape(w.shape[0], -1)
            z = get(prefix + ".weight_zero_point").float().reshape(w.shape[0], -1) \
                if has(prefix + ".weight_zero_point") else 0.0
            return (w.float() - z) * s
    return None


# ----------------------------------------------------------------------------- whole models
LINEAR_SUFFIXES = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                   "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


@torch.no_grad()
def calibrate(model, prompts: List[List[int]], keep_inputs: bool = True, max_rows: int = 4096) -> CalibrationCollector:
    """Runs the dense fp32 forward (a tensor-parallel size 1 CPU model) over the calibration
    prompts and records every linear layer's input under its HF name."""
    from rusteeze_b200.models.naive import naive_logits
    col = CalibrationCollector(keep_inputs, max_rows)
    for p in prompts:
        naive_logits(model, p, observer=col.record)
    return col


@torch.no_grad()
def quantize_model_checkpoint(model, out_dir: str, cfg: QuantConfig, prompts: Optional[List[List[int]]] = None,
                              stats: Optional[QuantStats] = None) -> Dict[str, torch.Tensor]:
    """Writes an HF checkpoint of `model` (a dense, tensor-parallel size 1 CPU model) with
    its attention and MLP linears in cfg.method's integer format -- gptq / awq (grouped
    4-bit, calibrated on `prompts`) or int8 (per-channel weight-only) -- and everything
    else as is; config.json carries the matching `quantization_config`."""
    import json
    import os
    from rusteeze_b200.models.loader import save_hf_checkpoint
    if cfg.method not in ("gptq", "awq", "int8"):
        raise ValueError("quantized checkpoints are written as gptq, awq or int8")
    save_hf_checkpoint(model, out_dir)
    from safetensors.torch import load_file, save_file
    files = sorted(f for f in os.listdir(out_dir) if f.endswith(".safetensors"))
    tensors: Dict[str, torch.Tensor] = {}
    for f in files:
        tensors.update(load_file(os.path.join(out_dir, f)))
        os.remove(os.path.join(out_dir, f))
    idx = os.path.join(out_dir, "model.safetensors.index.json")
    if os.path.exists(idx):
        os.remove(idx)
    col = calibrate(model, prompts) if cfg.method in ("gptq", "awq") else None
    stats = stats if stats is not None else QuantStats()
    out: Dict[str, torch.Tensor] = {}
    for name, w in tensors.items():
        prefix = name[:-len(".weight")] if name.endswith(".weight") else None
        if prefix is None or not prefix.endswith(LINEAR_SUFFIXES) or cfg.skips(prefix):
            out[name] = w
            continue
        W = w.float()
        if cfg.method == "int8":
            q, st = quantize_int8(W, per_channel=True, symmetric=True)
            out[prefix + ".weight"] = q
            out[prefix + ".weight_scale"] = st.scales.reshape(-1).float()
            stats.add(W, dequantize_int8(q, st), q.numel() + st.scales.numel() * 4)
            continue
        x = col.layer_inputs(prefix)
        if cfg.method == "gptq":
            codes, scales, zeros, g_idx = gptq_quantize(W, hessian(x), cfg.bits, cfg.group_size,
                                                        cfg.damp_percent, cfg.act_order, symmetric=False)
            # gptq_v2: zero points as they are (the v1 layout cannot store a zero point of 0)
            t = pack_gptq(codes, scales, zeros, g_idx, cfg.bits, v2=True)
            w_hat = unpack_gptq(t, cfg.bits, v2=True)
        else:
            codes, st, s = awq_quantize(W, x, cfg.bits, cfg.group_size)
            # s folded into the stored scales: w_hat = (Q(W s) / s), per input column --
            # kept exact by dividing each group's dequantized columns at load (s is saved)
            t = pack_awq(codes, st.scales, st.zero_points, cfg.bits)
            t["input_scale"] = s.to(torch.float32)
            w_hat = unpack_awq(t, cfg.bits) / s
        for k, v in t.items():
            out[prefix + "." + k] = v
        stats.add(W, w_hat, sum(v.numel() * v.element_size() for v in t.values()))
    save_file(out, os.path.join(out_dir, "model.safetensors"))
    with open(os.path.join(out_dir, "config.json")) as f:
        hf = json.load(f)
    hf["quantization_config"] = ({"quant_method": "int8", "bits": 8} if cfg.method == "int8" else
                                 {"quant_method": cfg.method, "bits": cfg.bits, "group_size": cfg.group_size,
                                  "desc_act": bool(cfg.act_order), "sym": False,
                                  **({"checkpoint_format": "gptq_v2"} if cfg.method == "gptq" else
                                     {"zero_point": True, "version": "gemm"})})
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(hf, f, indent=2)
    return out
