"""Typed configuration: defaults < file (YAML/TOML/JSON) < RUSTEEZE_* env < CLI.

Tree and knob names follow the reference's crates/rusteeze-config
(`Config {model, server, engine, logging, metrics}`, cfg/lib.rs:40-91;
model knobs cfg/model.rs:8-64; server knobs cfg/server.rs:9-58 incl. CORS,
TLS and rate limits; engine knobs cfg/engine.rs:7-81 incl. scheduling,
sampling defaults and speculative decoding) and config.example.yaml.  The
reference also carries a second, unused tree in crates/rusteeze-core/src/
config.rs; its extra knobs (cache_dtype, custom all-reduce) are folded in
here.  B200-specific knobs added: expert_parallel_size, comm_backend
(nccl | fused), kv_cache_dtype, quantization fp8_block, CUDA-graph buckets,
num_gpu_blocks override, model presets for random-init benchmarks.
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

from rusteeze_b200.core.errors import ConfigError


@dataclass
class QuantizationConfig:
    method: str = "none"        # none | fp8_block (fp8 / fp8_e4m3 accepted as aliases)
    bits: int = 8
    group_size: int = 128
    scale_format: str = "ue8m0"   # ue8m0 (power-of-two, applied in the MMA) | fp32 (applied per K block)


@dataclass
class ModelSection:
    path: Optional[str] = None          # local HF-layout directory
    preset: Optional[str] = None        # named random-init architecture (e.g. llama-3-8b)
    name: Optional[str] = None          # served model name
    revision: str = "main"
    dtype: str = "auto"                 # auto | float32 | float16 | bfloat16
    device: str = "auto"                # auto | cpu | cuda | cuda:N
    max_model_len: Optional[int] = None
    trust_remote_code: bool = False
    use_mmap: bool = True
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    expert_parallel_size: int = 1
    data_parallel_size: int = 1
    quantization: Optional[QuantizationConfig] = None
    tokenizer: Optional[str] = None
    chat_template: Optional[str] = None
    seed: int = 0

    def served_name(self) -> str:
        return self.name or self.preset or (os.path.basename(self.path.rstrip("/")) if self.path else "model")


@dataclass
class CorsConfig:
    enabled: bool = True
    allowed_origins: List[str] = field(default_factory=lambda: ["*"])
    allowed_methods: List[str] = field(default_factory=lambda: ["GET", "POST", "OPTIONS"])
    allowed_headers: List[str] = field(default_factory=lambda: ["Content-Type", "Authorization"])
    max_age: int = 86400


@dataclass
class TlsConfig:
    cert_path: Optional[str] = None
    key_path: Optional[str] = None


@dataclass
class RateLimitConfig:
    enabled: bool = False
    requests_per_minute: int = 60
    requests_per_day: Optional[int] = None
    tokens_per_minute: Optional[int] = None   # prompt + completion tokens per key
    tokens_per_day: Optional[int] = None
    burst: int = 10
    by: str = "api_key"                 # api_key | ip


@dataclass
class ServerSection:
    host: str = "0.0.0.0"
    port: int = 8000
    api_key: Optional[str] = None
    timeout_seconds: float = 300.0
    max_connections: int = 10000
    keep_alive_seconds: float = 75.0
    compression: bool = True
    max_body_bytes: int = 32 * 1024 * 1024
    workers: int = 1
    cors: CorsConfig = field(default_factory=CorsConfig)
    tls: Optional[TlsConfig] = None
    rate_limit: Optional[RateLimitConfig] = None
    metrics_port: Optional[int] = None
    router_policy: str = "least_loaded"    # data-parallel replicas: least_loaded | round_robin | random | prefix_affinity
    # a chat request's own Jinja `chat_template` runs only when this is set: the sandbox
    # stops code execution, not templates built to loop or allocate without bound
    trust_request_chat_template: bool = False


@dataclass
class SchedulingSection:
    policy: str = "fcfs"                # fcfs | sjf | priority
    enable_preemption: bool = True
    preemption_mode: str = "recompute"  # recompute | swap
    max_waiting_time_seconds: float = 60.0
    delay_factor: float = 0.0


@dataclass
class SamplingDefaults:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    max_tokens: int = 256
    repetition_penalty: float = 1.0


@dataclass
class SpeculativeSection:
    # proposer (crates/rusteeze-core/src/config.rs:635-645): "draft" (a draft model, or the
    # target itself when neither field below is set) | "ngram" (prompt lookup: no model)
    method: str = "draft"
    draft_model: Optional[str] = None    # HF dir of the draft model
    draft_preset: Optional[str] = None   # or a random-init preset (e.g. llama-3.2-1b)
    num_speculative_tokens: int = 4
    ngram_max: int = 4                   # longest suffix the n-gram proposer looks up
    ngram_min: int = 1                   # shortest
    acceptance_threshold: float = 0.9    # accepted for config parity; verification is exact


@dataclass
class EngineSection:
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    block_size: int = 16
    gpu_memory_utilization: float = 0.9
    num_gpu_blocks: Optional[int] = None      # override the memory-derived count
    swap_space_gb: float = 4.0
    kv_cache_dtype: str = "auto"              # auto (= model dtype) | fp8 (= fp8_e4m3) | fp8_e4m3 | fp8_e5m2
    enable_prefix_caching: bool = False
    enable_chunked_prefill: bool = False
    enforce_eager: bool = False               # disable CUDA graphs
    async_scheduling: bool = True             # overlap host scheduling / output processing with the GPU step
    cuda_graph_max_batch: Optional[int] = None
    comm_backend: str = "fused"               # nccl | fused (peer-memory kernels)
    request_timeout_seconds: float = 600.0
    scheduling: SchedulingSection = field(default_factory=SchedulingSection)
    sampling: SamplingDefaults = field(default_factory=SamplingDefaults)
    speculative: Optional[SpeculativeSection] = None


@dataclass
class LoggingSection:
    level: str = "info"
    format: str = "pretty"      # pretty | compact | json
    file: Optional[str] = None
    request_logging: bool = True


@dataclass
class PushGatewaySection:
    url: str = ""                        # e.g. http://pushgateway:9091
    job: str = "rusteeze"
    instance: Optional[str] = None
    interval_seconds: float = 15.0


@dataclass
class MetricsSection:
    enabled: bool = True
    path: str = "/metrics"
    prometheus: bool = True
    latency_buckets: List[float] = field(default_factory=lambda: [
        0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0, 60.0])
    push_gateway: Optional[PushGatewaySection] = None


@dataclass
class Config:
    model: ModelSection = field(default_factory=ModelSection)
    server: ServerSection = field(default_factory=ServerSection)
    engine: EngineSection = field(default_factory=EngineSection)
    logging: LoggingSection = field(default_factory=LoggingSection)
    metrics: MetricsSection = field(default_factory=MetricsSection)

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


# ----------------------------------------------------------------------------- (de)serialisation
def _from_dict(cls, data: Any):
    if data is None:
        return None
    if not dataclasses.is_dataclass(cls):
        return data
    if not isinstance(data, dict):
        raise ConfigError(f"expected a mapping for {cls.__name__}, got {type(data).__name__}")
    hints = {f.name: f for f in dataclasses.fields(cls)}
    kw = {}
    for k, v in data.items():
        if k not in hints:
            raise ConfigError(f"unknown config key {cls.__name__}.{k}")
        kw[k] = _convert(hints[k].type, v, f"{cls.__name__}.{k}")
    return cls(**kw)


_SECTION_TYPES = {
    "QuantizationConfig": QuantizationConfig, "CorsConfig": CorsConfig, "TlsConfig": TlsConfig,
    "RateLimitConfig": RateLimitConfig, "SchedulingSection": SchedulingSection,
    "SamplingDefaults": SamplingDefaults, "SpeculativeSection": SpeculativeSection,
    "ModelSection": ModelSection, "ServerSection": ServerSection, "EngineSection": EngineSection,
    "LoggingSection": LoggingSection, "MetricsSection": MetricsSection, "PushGatewaySection": PushGatewaySection,
}


def _convert(tp, v, where: str = "value"):
    """Checks a file or override value against the field's annotation: sections
    recurse; int / float / bool / str / List[...] fields get that type or a
    ConfigError naming the key (numeric strings, as environment variables give them,
    are accepted for numbers)."""
    t = tp if isinstance(tp, str) else getattr(tp, "__name__", str(tp))
    for name, cls in _SECTION_TYPES.items():
        if name in t:
            return _from_dict(cls, v)
    optional = t.startswith("Optional[")
    base = t[len("Optional["):-1] if optional else t
    if v is None:
        if optional:
            return None
        raise ConfigError(f"{where} must not be null")
    if base.startswith("List["):
        if not isinstance(v, (list, tuple)):
            raise ConfigError(f"{where} must be a list, got {type(v).__name__}")
        return [_convert(base[5:-1], x, f"{where}[{i}]") for i, x in enumerate(v)]
    if base == "bool":
        if isinstance(v, bool):
            return v
        if isinstance(v, str) and v.lower() in ("true", "false", "1", "0", "yes", "no"):
            return v.lower() in ("true", "1", "yes")
        raise ConfigError(f"{where} must be true or false, got {v!r}")
    if base in ("int", "float"):
        if isinstance(v, str):
            try:
                v = float(v) if base == "float" or any(c in v for c in ".eE") else int(v)
            except ValueError:
                raise ConfigError(f"{where} must be a number, got {v!r}") from None
        if isinstance(v, bool) or not isinstance(v, (int, float)):
            raise ConfigError(f"{where} must be a number, got {v!r}")
        if base == "int":
            if isinstance(v, float) and not v.is_integer():
                raise ConfigError(f"{where} must be an integer, got {v!r}")
            return int(v)
        return float(v)
    if base == "str":
        if isinstance(v, str):
            return v
        if isinstance(v, (int, float)) and not isinstance(v, bool):
            return str(v)              # e.g. an all-digit API key written unquoted
        raise ConfigError(f"{where} must be a string, got {v!r}")
    return v


def config_from_dict(d: Dict[str, Any]) -> Config:
    cfg = _from_dict(Config, d or {})
    return cfg


def merge_dict(base: Dict[str, Any], over: Dict[str, Any]) -> Dict[str, Any]:
    out = dict(base)
    for k, v in over.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = merge_dict(out[k], v)
        else:
            out[k] = v
    return out
