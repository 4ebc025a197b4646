"""HF `config.json` parsing into one typed `ModelConfig`, plus the named
benchmark architectures.

Field set and defaults follow crates/rusteeze-model/src/config.rs:123-230
(ModelConfig: GQA heads, explicit head_dim, rope_scaling, sliding_window,
num_experts / num_experts_per_tok, tie_word_embeddings defaulting to true
:187-189, EOS single-or-list :235-258, RoPE scaling :262-285).  Unlike the
reference, every field an architecture needs at runtime (Gemma's embedding
scale and soft-caps, Phi3's fused checkpoint tensors, Qwen2's QKV bias) is a
first-class attribute here.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field, asdict
from typing import List, Optional

from rusteeze_b200.core.errors import ConfigError
from rusteeze_b200.core.types import ModelArchitecture


@dataclass
class RopeScaling:
    type: str = "none"                 # none | linear | dynamic | llama3
    factor: float = 1.0
    original_max_position_embeddings: Optional[int] = None
    low_freq_factor: Optional[float] = None
    high_freq_factor: Optional[float] = None


@dataclass
class ModelConfig:
    architecture: ModelArchitecture = ModelArchitecture.LLAMA
    hidden_size: int = 4096
    intermediate_size: int = 11008
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: Optional[int] = None
    head_dim: Optional[int] = None
    vocab_size: int = 32000
    max_position_embeddings: int = 4096
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: Optional[RopeScaling] = None
    sliding_window: Optional[int] = None
    hidden_act: str = "silu"
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    mlp_bias: bool = False
    num_local_experts: int = 0
    num_experts_per_tok: int = 0
    bos_token_id: Optional[int] = 1
    eos_token_id: List[int] = field(default_factory=lambda: [2])
    pad_token_id: Optional[int] = None
    torch_dtype: str = "bfloat16"
    # Gemma / Gemma2 specifics
    attn_logit_softcapping: Optional[float] = None
    final_logit_softcapping: Optional[float] = None
    query_pre_attn_scalar: Optional[float] = None
    sliding_window_pattern: int = 0    # gemma2: every 2nd layer (even index) is local
    # positions: "rope" (rotary q/k) or "alibi" (no rotation; a per-head linear bias on the
    # attention logits, crates/rusteeze-tensor/src/attention.rs:33-34,341-390)
    position_embedding: str = "rope"
    name: str = "custom"

    def __post_init__(self) -> None:
        if self.num_key_value_heads is None:
            self.num_key_value_heads = self.num_attention_heads
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_attention_heads
        if isinstance(self.architecture, str):
            self.architecture = ModelArchitecture(self.architecture)
        if isinstance(self.rope_scaling, dict):
            self.rope_scaling = _parse_rope_scaling(self.rope_scaling)
        if isinstance(self.eos_token_id, int):
            self.eos_token_id = [self.eos_token_id]
        self.validate()

    # ------------------------------------------------------------------
    @property
    def is_moe(self) -> bool:
        return self.num_local_experts > 0

    @property
    def is_gqa(self) -> bool:
        return self.num_key_value_heads < self.num_attention_heads

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def embed_scale(self) -> float:
        if self.architecture in (ModelArchitecture.GEMMA, ModelArchitecture.GEMMA2):
            return float(self.hidden_size) ** 0.5
        return 1.0

    @property
    def norm_offset(self) -> float:
        """Gemma stores RMSNorm weights as (w - 1)."""
        return 1.0 if self.architecture in (ModelArchitecture.GEMMA, ModelArchitecture.GEMMA2) else 0.0

    @property
    def attn_scale(self) -> float:
        if self.query_pre_attn_scalar:
            return float(self.query_pre_attn_scalar) ** -0.5
        return float(self.head_dim) ** -0.5

    def layer_sliding_window(self, layer_idx: int) -> Optional[int]:
        if self.architecture == ModelArchitecture.GEMMA2:
            return self.sliding_window if layer_idx % 2 == 0 else None
        return self.sliding_window

    def num_params(self) -> int:
        h, i, v = self.hidden_size, self.intermediate_size, self.vocab_size
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        mlp = 3 * h * i * max(1, self.num_local_experts) + (h * self.num_local_experts)
        per_layer = attn + mlp + 2 * h
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_hidden_layers * per_layer + emb + h

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return 2 * self.num_hidden_layers * self.kv_size * dtype_bytes

    def validate(self) -> None:
        if self.num_attention_heads % self.num_key_value_heads:
            raise ConfigError("num_attention_heads must be a multiple of num_key_value_heads")
        if self.head_dim % 16:
            raise ConfigError(f"head_dim {self.head_dim} must be a multiple of 16")
        if self.is_moe and not 0 < self.num_experts_per_tok <= self.num_local_experts:
            raise ConfigError("num_experts_per_tok must be in [1, num_local_experts]")
        if self.position_embedding not in ("rope", "alibi"):
            raise ConfigError(f"position_embedding must be rope or alibi, got {self.position_embedding!r}")

    @property
    def use_alibi(self) -> bool:
        return self.position_embedding == "alibi"

    def to_dict(self) -> dict:
        d = asdict(self)
        d["architecture"] = self.architecture.value
        return d

    # ------------------------------------------------------------------
    @classmethod
    def from_hf_dict(cls, d: dict) -> "ModelConfig":
        arch = ModelArchitecture.from_hf(d.get("model_type"), d.get("architectures"))
        eos = d.get("eos_token_id", 2)
        if eos is None:
            eos = []
        kw = dict(
            architecture=arch,
            hidden_size=d["hidden_size"],
            intermediate_size=d["intermediate_size"],
            num_hidden_layers=d["num_hidden_layers"],
            num_attention_heads=d["num_attention_heads"],
            num_key_value_heads=d.get("num_key_value_heads"),
            head_dim=d.get("head_dim"),
            vocab_size=d["vocab_size"],
            max_position_embeddings=d.get("max_position_embeddings", 4096),
            rms_norm_eps=d.get("rms_norm_eps", 1e-6),
            rope_theta=d.get("rope_theta", 10000.0),
            rope_scaling=_parse_rope_scaling(d.get("rope_scaling")),
            sliding_window=d.get("sliding_window"),
            hidden_act=d.get("hidden_act", d.get("hidden_activation", "silu")) or "silu",
            tie_word_embeddings=d.get("tie_word_embeddings",
                                      arch in (ModelArchitecture.GEMMA, ModelArchitecture.GEMMA2)),
            attention_bias=d.get("attention_bias", arch == ModelArchitecture.QWEN2),
            mlp_bias=d.get("mlp_bias", False),
            num_local_experts=d.get("num_local_experts", d.get("num_experts", 0)) or 0,
            num_experts_per_tok=d.get("num_experts_per_tok", 0) or 0,
            bos_token_id=d.get("bos_token_id"),
            eos_token_id=eos if isinstance(eos, list) else [eos],
            pad_token_id=d.get("pad_token_id"),
            torch_dtype=d.get("torch_dtype", "bfloat16") or "bfloat16",
            attn_logit_softcapping=d.get("attn_logit_softcapping"),
            final_logit_softcapping=d.get("final_logit_softcapping"),
            query_pre_attn_scalar=d.get("query_pre_attn_scalar"),
            position_embedding=("alibi" if d.get("alibi") or d.get("position_embedding_type") == "alibi"
                                else "rope"),
            name=d.get("_name_or_path", "hf"),
        )
        if arch == ModelArchitecture.QWEN2 and not d.get("use_sliding_window", False):
            kw["sliding_window"] = None
        return cls(**kw)

    @classmethod
    def from_json_file(cls, path: str) -> "ModelConfig":
        if os.path.isdir(path):
            path = os.path.join(path, "config.json")
        with open(path) as f:
            return cls.from_hf_dict(json.load(f))

    def to_hf_dict(self) -> dict:
        d = {
            "model_type": self.architecture.value,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "vocab_size": self.vocab_size,
            "max_position_embeddings": self.max_position_embeddings,
            "rms_norm_eps": self.rms_norm_eps,
            "rope_theta": self.rope_theta,
            "sliding_window": self.sliding_window,
            "hidden_act": self.hidden_act,
            "tie_word_embeddings": self.tie_word_embeddings,
            "attention_bias": self.attention_bias,
            "bos_token_id": self.bos_token_id,
            "eos_token_id": self.eos_token_id,
            "torch_dtype": self.torch_dtype,
        }
        if self.rope_scaling is not None:
            d["rope_scaling"] = {"rope_type": self.rope_scaling.type, **{
                k: v for k, v in asdict(self.rope_scaling).items() if k != "type" and v is not None}}
        if self.is_moe:
            d["num_local_experts"] = self.num_local_experts
            d["num_experts_per_tok"] = self.num_experts_per_tok
        for k in ("attn_logit_softcapping", "final_logit_softcapping", "query_pre_attn_scalar"):
            if getattr(self, k) is not None:
                d[k] = getattr(self, k)
        if self.use_alibi:
            d["alibi"] = True
        return d


def _parse_rope_scaling(d) -> Optional[RopeScaling]:
    if not d:
        return None
    if isinstance(d, RopeScaling):
        return d
    t = d.get("rope_type", d.get("type", "linear"))
    if t == "default":
        return None
    return RopeScaling(type=t, factor=float(d.get("factor", 1.0)),
                       original_max_position_embeddings=d.get("original_max_position_embeddings"),
                       low_freq_factor=d.get("low_freq_factor"),
                       high_freq_factor=d.get("high_freq_factor"))


# ----------------------------------------------------------------------------
# Named architectures used by the benchmarks and tests (random-init weights).
# ----------------------------------------------------------------------------
def _preset(**kw) -> ModelConfig:
    return ModelConfig(**kw)


PRESETS = {
    # 2 layers, hidden 256, 4q/2kv (head_dim 64), SwiGLU 688, vocab 32000
    "tiny-llama": lambda: _preset(name="tiny-llama", hidden_size=256, intermediate_size=688,
                                  num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                                  vocab_size=32000, rms_norm_eps=1e-5, rope_theta=10000.0,
                                  max_position_embeddings=2048),
    # Mixtral-shaped MoE for harness tests: 2 layers, 4 experts (top-2), 4q/2kv
    "tiny-mixtral": lambda: _preset(name="tiny-mixtral", architecture=ModelArchitecture.MIXTRAL, hidden_size=256,
                                    intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                                    num_key_value_heads=2, vocab_size=32000, rms_norm_eps=1e-5, rope_theta=1e6,
                                    num_local_experts=4, num_experts_per_tok=2, max_position_embeddings=2048),
    "llama-2-7b": lambda: _preset(name="llama-2-7b", hidden_size=4096, intermediate_size=11008,
                                  num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=32,
                                  vocab_size=32000, rms_norm_eps=1e-5, rope_theta=10000.0,
                                  max_position_embeddings=4096),
    "llama-3-8b": lambda: _preset(name="llama-3-8b", hidden_size=4096, intermediate_size=14336,
                                  num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                                  vocab_size=128256, rms_norm_eps=1e-5, rope_theta=500000.0,
                                  max_position_embeddings=8192, bos_token_id=128000,
                                  eos_token_id=[128001, 128009]),
    "llama-3-70b": lambda: _preset(name="llama-3-70b", hidden_size=8192, intermediate_size=28672,
                                   num_hidden_layers=80, num_attention_heads=64, num_key_value_heads=8,
                                   vocab_size=128256, rms_norm_eps=1e-5, rope_theta=500000.0,
                                   max_position_embeddings=8192, bos_token_id=128000,
                                   eos_token_id=[128001, 128009]),
    "llama-3.2-1b": lambda: _preset(name="llama-3.2-1b", hidden_size=2048, intermediate_size=8192,
                                    num_hidden_layers=16, num_attention_heads=32, num_key_value_heads=8,
                                    head_dim=64, vocab_size=128256, rms_norm_eps=1e-5,
                                    rope_theta=500000.0, max_position_embeddings=8192,
                                    tie_word_embeddings=True, bos_token_id=128000,
                                    eos_token_id=[128001, 128009]),
    "mistral-7b": lambda: _preset(name="mistral-7b", architecture=ModelArchitecture.MISTRAL,
                                  hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                                  num_attention_heads=32, num_key_value_heads=8, vocab_size=32000,
                                  rms_norm_eps=1e-5, rope_theta=10000.0, sliding_window=4096,
                                  max_position_embeddings=32768),
    "mixtral-8x7b": lambda: _preset(name="mixtral-8x7b", architecture=ModelArchitecture.MIXTRAL,
                                    hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                                    num_attention_heads=32, num_key_value_heads=8, vocab_size=32000,
                                    rms_norm_eps=1e-5, rope_theta=1e6, num_local_experts=8,
                                    num_experts_per_tok=2, max_position_embeddings=32768),
}


def get_preset(name: str) -> ModelConfig:
    try:
        return PRESETS[name]()
    except KeyError:
        raise ConfigError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}") from None


def tiny_variant(arch: ModelArchitecture, **kw) -> ModelConfig:
    """Small config of any architecture for CPU oracle tests."""
    base = dict(name=f"tiny-{arch.value}", architecture=arch, hidden_size=128, intermediate_size=256,
                num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, vocab_size=512,
                rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=1024)
    if arch == ModelArchitecture.MIXTRAL:
        base.update(num_local_experts=4, num_experts_per_tok=2)
    if arch == ModelArchitecture.MISTRAL:
        base.update(sliding_window=24)
    if arch == ModelArchitecture.QWEN2:
        base.update(attention_bias=True)
    if arch in (ModelArchitecture.GEMMA, ModelArchitecture.GEMMA2):
        base.update(hidden_act="gelu_pytorch_tanh", tie_word_embeddings=True, head_dim=32)
    if arch == ModelArchitecture.GEMMA2:
        base.update(attn_logit_softcapping=50.0, final_logit_softcapping=30.0,
                    query_pre_attn_scalar=32, sliding_window=24)
    base.update(kw)
    return ModelConfig(**base)
