"""Checkpoint loading, tensor-parallel slicing, and seeded random init.

Checkpoint format is the HF layout the reference reads
(crates/rusteeze-model/src/loader.rs): `config.json` + one or more
`*.safetensors` files (sharded names `model-0000N-of-0000M.safetensors`,
loader.rs:91-97, with an optional `model.safetensors.index.json`,
loader.rs:432-457), opened memory-mapped (loader.rs:263-300).

Differences by design:
  * Each rank reads only the slice it owns (column split of q/k/v and
    gate/up by head/column, row split of o/down, vocab split of the
    embedding and LM head, experts by EP rank) -- the reference's
    `WeightShard`/`shard_tensor` helpers (crates/rusteeze-model/src/
    weights.rs:345-399) were never used by its models.
  * q/k/v and gate/up are fused at load (weights.rs:299-341 has the same
    helpers, unused) into the K-major layouts the GEMM kernel consumes.
  * Checkpoint tensors are used as stored; HF Llama has no projection
    biases, so none are expected (the reference's candle `linear` also
    asks for a bias tensor, common.rs:210-217).
  * `init_random` gives every benchmark model N(0, 0.02) weights from a
    seed, identical for any TP size (each rank draws the full logical
    tensor with a per-tensor seed and keeps its slice).
"""
from __future__ import annotations

import glob
import hashlib
import json
import os
from typing import Callable, Dict, Iterable, Optional, Tuple

import torch

from rusteeze_b200.core.errors import ModelLoadError
from rusteeze_b200.core.types import ModelArchitecture
from rusteeze_b200.models.config import ModelConfig
from rusteeze_b200.models.decoder import DecoderLM


# ----------------------------------------------------------------------------- shard specs
def _rows(t: torch.Tensor, lo: int, hi: int) -> torch.Tensor:
    return t[lo:hi]


def _kv_head_range(model: DecoderLM) -> Tuple[int, int]:
    cfg, tps, tpr = model.cfg, model.tp.size, model.tp.rank
    if cfg.num_key_value_heads >= tps:
        per = cfg.num_key_value_heads // tps
        return tpr * per, (tpr + 1) * per
    h = tpr * cfg.num_key_value_heads // tps
    return h, h + 1


def shard_qkv(model: DecoderLM, full: torch.Tensor) -> torch.Tensor:
    """full: fused [q_all | k_all | v_all] along dim 0 -> this rank's [q | k | v]."""
    cfg, D = model.cfg, model.cfg.head_dim
    qs, kvs = cfg.q_size, cfg.kv_size
    r = model.tp.rank
    q = full[r * model.hq * D:(r + 1) * model.hq * D]
    a, b = _kv_head_range(model)
    k = full[qs + a * D: qs + b * D]
    v = full[qs + kvs + a * D: qs + kvs + b * D]
    return torch.cat([q, k, v], dim=0)


def shard_gate_up(model: DecoderLM, full: torch.Tensor) -> torch.Tensor:
    I = model.cfg.intermediate_size
    r, il = model.tp.rank, model.inter
    return torch.cat([full[r * il:(r + 1) * il], full[I + r * il: I + (r + 1) * il]], dim=0)


def shard_cols(model: DecoderLM, full: torch.Tensor, width: int) -> torch.Tensor:
    r = model.tp.rank
    return full[:, r * width:(r + 1) * width]


def shard_vocab(model: DecoderLM, full: torch.Tensor) -> torch.Tensor:
    V = full.shape[0]
    lo, hi = model.vocab_lo, model.vocab_hi
    out = full.new_zeros(hi - lo, full.shape[1])
    n = max(0, min(hi, V) - lo)
    if n:
        out[:n] = full[lo:lo + n]
    return out


def logical_params(model: DecoderLM) -> Iterable[Tuple[str, Tuple[int, ...], Callable, str]]:
    """(internal name, full logical shape, full->local slicer, init kind)."""
    cfg = model.cfg
    H, D, V = cfg.hidden_size, cfg.head_dim, cfg.vocab_size
    I = cfg.intermediate_size
    ident = lambda t: t  # noqa: E731
    yield "embed", (V, H), lambda t: shard_vocab(model, t), "normal"
    for i, L in enumerate(model.layers):
        p = f"layers.{i}."
        yield p + "input_norm", (H,), ident, "norm"
        yield p + "post_attn_norm", (H,), ident, "norm"
        yield p + "qkv", (cfg.q_size + 2 * cfg.kv_size, H), lambda t: shard_qkv(model, t), "normal"
        if L.qkv_bias is not None:
            yield p + "qkv_bias", (cfg.q_size + 2 * cfg.kv_size,), lambda t: shard_qkv(model, t), "zero"
        yield p + "o", (H, cfg.q_size), lambda t: shard_cols(model, t, model.hq * D), "normal"
        if model.is_gemma2:
            yield p + "pre_ff_norm", (H,), ident, "norm"
            yield p + "post_ff_norm", (H,), ident, "norm"
        if cfg.is_moe:
            E = cfg.num_local_experts
            yield p + "router", (E, H), ident, "normal"
            yield p + "w13", (E, 2 * I, H), lambda t: t[model.e_lo:model.e_hi], "normal"
            yield p + "w2", (E, H, I), lambda t: t[model.e_lo:model.e_hi], "normal"
        else:
            yield p + "gate_up", (2 * I, H), lambda t: shard_gate_up(model, t), "normal"
            yield p + "down", (H, I), lambda t: shard_cols(model, t, model.inter), "normal"
    yield "norm", (H,), ident, "norm"
    if model.lm_head is not None:
        yield "lm_head", (V, H), lambda t: shard_vocab(model, t), "normal"


def _param(model: DecoderLM, name: str) -> torch.nn.Parameter:
    obj = model
    for part in name.split("."):
        obj = obj[int(part)] if part.isdigit() else getattr(obj, part)
    return obj


def _seed_for(name: str, seed: int) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:7], "little")


@torch.no_grad()
def init_random(model: DecoderLM, seed: int = 0, std: float = 0.02) -> DecoderLM:
    """N(0, std) weights, unit norms (zero for Gemma's (1+w) norms), zero biases."""
    dev = model.device
    for name, shape, slicer, kind in logical_params(model):
        p = _param(model, name)
        if kind == "norm":
            p.fill_(0.0 if model.cfg.norm_offset else 1.0)
            continue
        if kind == "zero":
            p.zero_()
            continue
        g = torch.Generator(device=dev)
        g.manual_seed(_seed_for(name, seed))
        if len(shape) == 3:
            # experts: draw per expert so the slice never materialises all of them
            for j, e in enumerate(range(model.e_lo, model.e_hi)):
                g.manual_seed(_seed_for(f"{name}.{e}", seed))
                p[j].copy_(torch.randn(shape[1:], generator=g, device=dev, dtype=torch.float32)
                           .mul_(std).to(p.dtype))
            continue
        full = torch.empty(shape, device=dev, dtype=p.dtype)
        # bf16 randn in chunks keeps peak memory at one extra full tensor
        rows = max(1, (1 << 26) // max(1, full[0].numel()))
        for a in range(0, shape[0], rows):
            full[a:a + rows] = torch.randn((min(rows, shape[0] - a),) + tuple(shape[1:]), generator=g,
                                           device=dev, dtype=torch.float32).mul_(std).to(p.dtype)
        p.copy_(slicer(full))
        del full
    return model


# ----------------------------------------------------------------------------- HF checkpoints
def discover_weight_files(model_dir: str):
    """safetensors (preferred; sharded via model.safetensors.index.json) or, as
    the reference's loader also accepts, PyTorch `pytorch_model*.bin` files
    (sharded via pytorch_model.bin.index.json)."""
    for index_name, pattern in (("model.safetensors.index.json", "*.safetensors"),
                                ("pytorch_model.bin.index.json", "pytorch_model*.bin")):
        idx = os.path.join(model_dir, index_name)
        if os.path.exists(idx):
            with open(idx) as f:
                files = sorted(set(json.load(f)["weight_map"].values()))
            return [os.path.join(model_dir, x) for x in files]
        files = sorted(glob.glob(os.path.join(model_dir, pattern)))
        if files:
            return files
    raise ModelLoadError(f"no *.safetensors or pytorch_model*.bin files in {model_dir}")


class _TensorIndex:
    """Checkpoint tensors by name.  With `quant` (an integer `quantization_config`: gptq, awq,
    int8 weight-only), a layer's `<prefix>.weight` is rebuilt from its integer tensors."""

    def __init__(self, files, quant: Optional[dict] = None):
        self.quant = quant
        self.handles = []
        for f in files:
            if f.endswith(".safetensors"):
                from safetensors import safe_open
                self.handles.append(safe_open(f, framework="pt", device="cpu"))
            else:
                # PyTorch pickles are loaded tensor-only (no code execution) and memory-mapped
                self.handles.append(torch.load(f, map_location="cpu", weights_only=True, mmap=True))
        self.where: Dict[str, int] = {}
        for i, h in enumerate(self.handles):
            for k in h.keys():
                self.where[k] = i

    def has(self, k: str) -> bool:
        if k in self.where:
            return True
        return bool(self.quant) and k.endswith(".weight") and k[:-7] + ".qweight" in self.where

    def _raw(self, k: str) -> torch.Tensor:
        if k not in self.where:
            raise ModelLoadError(f"missing weight {k}")
        h = self.handles[self.where[k]]
        return h[k] if isinstance(h, dict) else h.get_tensor(k)

    def get(self, k: str) -> torch.Tensor:
        if self.quant and k.endswith(".weight"):
            from rusteeze_b200.models.int_quant import dequantize_checkpoint_tensor
            w = dequantize_checkpoint_tensor(self._raw, lambda n: n in self.where, k[:-7], self.quant)
            if w is not None:
                return w
        return self._raw(k)


def _hf_full(ix: _TensorIndex, cfg: ModelConfig, name: str) -> torch.Tensor:
    """Build the full logical fused tensor for an internal name from HF tensors."""
    arch = cfg.architecture
    if name == "embed":
        return ix.get("model.embed_tokens.weight")
    if name == "norm":
        return ix.get("model.norm.weight")
    if name == "lm_head":
        return ix.get("lm_head.weight")
    _, i, leaf = name.split(".", 2)
    p = f"model.layers.{i}."
    if leaf == "input_norm":
        return ix.get(p + "input_layernorm.weight")
    if leaf == "post_attn_norm":
        return ix.get(p + "post_attention_layernorm.weight")
    if leaf == "pre_ff_norm":
        return ix.get(p + "pre_feedforward_layernorm.weight")
    if leaf == "post_ff_norm":
        return ix.get(p + "post_feedforward_layernorm.weight")
    if leaf in ("qkv", "qkv_bias"):
        suf = "weight" if leaf == "qkv" else "bias"
        if ix.has(p + f"self_attn.qkv_proj.{suf}"):
            return ix.get(p + f"self_attn.qkv_proj.{suf}")
        return torch.cat([ix.get(p + f"self_attn.{x}_proj.{suf}") for x in "qkv"], dim=0)
    if leaf == "o":
        return ix.get(p + "self_attn.o_proj.weight")
    if leaf == "gate_up":
        if ix.has(p + "mlp.gate_up_proj.weight"):
            return ix.get(p + "mlp.gate_up_proj.weight")
        return torch.cat([ix.get(p + "mlp.gate_proj.weight"), ix.get(p + "mlp.up_proj.weight")], 0)
    if leaf == "down":
        return ix.get(p + "mlp.down_proj.weight")
    if arch == ModelArchitecture.MIXTRAL:
        m = p + "block_sparse_moe."
        E = cfg.num_local_experts
        if leaf == "router":
            return ix.get(m + "gate.weight")
        if leaf == "w13":
            return torch.stack([torch.cat([ix.get(m + f"experts.{e}.w1.weight"),
                                           ix.get(m + f"experts.{e}.w3.weight")], 0) for e in range(E)])
        if leaf == "w2":
            return torch.stack([ix.get(m + f"experts.{e}.w2.weight") for e in range(E)])
    raise ModelLoadError(f"no HF mapping for {name} ({arch.value})")


def checkpoint_quantization(model_dir: str) -> Optional[dict]:
    """The integer `quantization_config` of a checkpoint's config.json (gptq, awq, int8), if
    any: such layers are dequantized to the model dtype while loading."""
    path = os.path.join(model_dir, "config.json")
    if not os.path.exists(path):
        return None
    from rusteeze_b200.models.int_quant import checkpoint_quant_config
    with open(path) as f:
        return checkpoint_quant_config(json.load(f))


@torch.no_grad()
def load_hf_weights(model: DecoderLM, model_dir: str) -> DecoderLM:
    ix = _TensorIndex(discover_weight_files(model_dir), checkpoint_quantization(model_dir))
    for name, shape, slicer, _kind in logical_params(model):
        full = _hf_full(ix, model.cfg, name)
        if tuple(full.shape) != tuple(shape):
            raise ModelLoadError(f"{name}: checkpoint shape {tuple(full.shape)} != expected {shape}")
        _param(model, name).copy_(slicer(full).to(model.dtype))
    return model


def save_hf_checkpoint(model: DecoderLM, out_dir: str, shard_bytes: int = 1 << 30) -> None:
    """Writes an unsharded (TP=1) model in HF layout; used by tests and the
    `download`-less offline workflow."""
    from safetensors.torch import save_file
    assert model.tp.size == 1
    cfg = model.cfg
    os.makedirs(out_dir, exist_ok=True)
    t: Dict[str, torch.Tensor] = {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.norm}
    if model.lm_head is not None:
        t["lm_head.weight"] = model.lm_head
    I = cfg.intermediate_size
    for i, L in enumerate(model.layers):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = L.input_norm
        t[p + "post_attention_layernorm.weight"] = L.post_attn_norm
        qs, kvs = cfg.q_size, cfg.kv_size
        t[p + "self_attn.q_proj.weight"] = L.qkv[:qs]
        t[p + "self_attn.k_proj.weight"] = L.qkv[qs:qs + kvs]
        t[p + "self_attn.v_proj.weight"] = L.qkv[qs + kvs:]
        if L.qkv_bias is not None:
            t[p + "self_attn.q_proj.bias"] = L.qkv_bias[:qs]
            t[p + "self_attn.k_proj.bias"] = L.qkv_bias[qs:qs + kvs]
            t[p + "self_attn.v_proj.bias"] = L.qkv_bias[qs + kvs:]
        t[p + "self_attn.o_proj.weight"] = L.o
        if model.is_gemma2:
            t[p + "pre_feedforward_layernorm.weight"] = L.pre_ff_norm
            t[p + "post_feedforward_layernorm.weight"] = L.post_ff_norm
        if cfg.is_moe:
            m = p + "block_sparse_moe."
            t[m + "gate.weight"] = L.router
            for e in range(cfg.num_local_experts):
                t[m + f"experts.{e}.w1.weight"] = L.w13[e, :I]
                t[m + f"experts.{e}.w3.weight"] = L.w13[e, I:]
                t[m + f"experts.{e}.w2.weight"] = L.w2[e]
        else:
            t[p + "mlp.gate_proj.weight"] = L.gate_up[:I]
            t[p + "mlp.up_proj.weight"] = L.gate_up[I:]
            t[p + "mlp.down_proj.weight"] = L.down
    t = {k: v.detach().contiguous().cpu() for k, v in t.items()}
    # shard into N files + index, like HF
    shards, cur, size = [], {}, 0
    for k in sorted(t):
        nb = t[k].numel() * t[k].element_size()
        if cur and size + nb > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t[k]
        size += nb
    shards.append(cur)
    wm = {}
    for j, sh in enumerate(shards):
        fn = f"model-{j + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(out_dir, fn))
        wm.update({k: fn for k in sh})
    with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg.to_hf_dict(), f, indent=1)


def build_model(cfg: ModelConfig, *, dtype=torch.bfloat16, device="cpu", tp=None,
                ep_rank: int = 0, ep_size: int = 1, model_dir: Optional[str] = None,
                seed: int = 0) -> DecoderLM:
    model = DecoderLM(cfg, dtype=dtype, device=device, tp=tp, ep_rank=ep_rank, ep_size=ep_size)
    if model_dir:
        load_hf_weights(model, model_dir)
    else:
        init_random(model, seed)
    return model.eval()


@torch.no_grad()
def to_cpu_fp32(model: DecoderLM) -> DecoderLM:
    """An fp32 CPU copy of a (possibly GPU-prepared) model with identical weights."""
    from rusteeze_b200.ops import deinterleave_gate_up
    out = DecoderLM(model.cfg, dtype=torch.float32, device="cpu", tp=None)
    for name, _shape, _slicer, _kind in logical_params(out):
        src = _param(model, name)
        if name.endswith("gate_up") and src.numel() == 0:
            src = deinterleave_gate_up(_param(model, name[:-len("gate_up")] + "gate_up_il"))
        if name.endswith("w13") and src.numel() == 0:
            il = _param(model, name + "_il")
            src = torch.stack([deinterleave_gate_up(il[e]) for e in range(il.shape[0])])
        _param(out, name).copy_(src.float().cpu())
    return out.eval()
