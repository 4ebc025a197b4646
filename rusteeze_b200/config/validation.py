"""Semantic validation of a loaded Config (crates/rusteeze-config/src/
validation.rs:7-195: dtype/device/TP/port/ranges; HF repo id vs local path)."""
from __future__ import annotations

import os
import re
from typing import List

from rusteeze_b200.core.errors import ConfigError

_DTYPES = {"auto", "float32", "float16", "bfloat16", "fp32", "fp16", "bf16"}
_DEVICE_RE = re.compile(r"^(auto|cpu|cuda(:\d+)?)$")
_HF_REPO_RE = re.compile(r"^[A-Za-z0-9_.-]+/[A-Za-z0-9_.-]+$")


def is_hf_repo_id(s: str) -> bool:
    return bool(_HF_REPO_RE.match(s)) and not os.path.exists(s)


def collect_errors(cfg) -> List[str]:
    e: List[str] = []
    m, s, g = cfg.model, cfg.server, cfg.engine
    if m.dtype not in _DTYPES:
        e.append(f"model.dtype must be one of {sorted(_DTYPES)}, got {m.dtype!r}")
    if not _DEVICE_RE.match(m.device):
        e.append(f"model.device must be auto|cpu|cuda|cuda:N (metal/vulkan are not supported), got {m.device!r}")
    for k in ("tensor_parallel_size", "expert_parallel_size"):
        v = getattr(m, k)
        if v < 1 or v & (v - 1):
            e.append(f"model.{k} must be a power of two >= 1, got {v}")
    if m.data_parallel_size < 1:
        e.append(f"model.data_parallel_size must be >= 1, got {m.data_parallel_size}")
    if m.data_parallel_size > 1 and m.tensor_parallel_size > 1:
        e.append("model.data_parallel_size > 1 serves tensor_parallel_size 1 replicas (one GPU each)")
    if m.data_parallel_size > 1 and m.device.startswith("cuda:"):
        e.append("model.device must be auto|cuda|cpu with data_parallel_size > 1 (replica i runs on cuda:i)")
    if s.router_policy not in ("least_loaded", "round_robin", "random", "prefix_affinity"):
        e.append("server.router_policy must be least_loaded|round_robin|random|prefix_affinity, "
                 f"got {s.router_policy!r}")
    if m.pipeline_parallel_size != 1:
        e.append("model.pipeline_parallel_size > 1 is not supported: one NVSwitch domain serves these "
                 "models with tensor/expert parallelism")
    if m.quantization is not None and m.quantization.method not in ("none", "fp8_block", "fp8", "fp8_e4m3"):
        e.append(f"model.quantization.method {m.quantization.method!r} unsupported (none | fp8_block)")
    if m.max_model_len is not None and m.max_model_len < 16:
        e.append("model.max_model_len must be >= 16")
    if not 0 < s.port < 65536:
        e.append(f"server.port out of range: {s.port}")
    if s.timeout_seconds <= 0:
        e.append("server.timeout_seconds must be > 0")
    if s.tls is not None and (not s.tls.cert_path or not s.tls.key_path):
        e.append("server.tls needs cert_path and key_path")
    rl = s.rate_limit
    if rl is not None and rl.enabled:
        if rl.requests_per_minute < 1:
            e.append(f"server.rate_limit.requests_per_minute must be >= 1, got {rl.requests_per_minute}")
        if rl.by not in ("api_key", "ip"):
            e.append(f"server.rate_limit.by must be api_key|ip, got {rl.by!r}")
        if rl.burst < 0:
            e.append(f"server.rate_limit.burst must be >= 0, got {rl.burst}")
        if rl.requests_per_day is not None and rl.requests_per_day < 1:
            e.append(f"server.rate_limit.requests_per_day must be >= 1, got {rl.requests_per_day}")
        for name in ("tokens_per_minute", "tokens_per_day"):
            v = getattr(rl, name)
            if v is not None and v < 1:
                e.append(f"server.rate_limit.{name} must be >= 1, got {v}")
    if g.max_num_seqs < 1:
        e.append("engine.max_num_seqs must be >= 1")
    if g.max_num_batched_tokens < g.max_num_seqs:
        e.append("engine.max_num_batched_tokens must be >= engine.max_num_seqs")
    if g.block_size != 16:
        e.append("engine.block_size must be 16 (the paged-attention kernels are built for 16-token blocks)")
    if not 0.0 < g.gpu_memory_utilization <= 1.0:
        e.append("engine.gpu_memory_utilization must be in (0, 1]")
    if g.swap_space_gb < 0:
        e.append("engine.swap_space_gb must be >= 0")
    if g.scheduling.policy not in ("fcfs", "sjf", "priority"):
        e.append(f"engine.scheduling.policy must be fcfs|sjf|priority, got {g.scheduling.policy!r}")
    if g.scheduling.preemption_mode not in ("recompute", "swap"):
        e.append("engine.scheduling.preemption_mode must be recompute|swap")
    if g.comm_backend not in ("nccl", "fused"):
        e.append("engine.comm_backend must be nccl|fused")
    if g.speculative is not None and not 1 <= g.speculative.num_speculative_tokens <= 16:
        e.append("engine.speculative.num_speculative_tokens must be in [1, 16]")
    if g.speculative is not None:
        sp = g.speculative
        if sp.method in ("medusa", "mlp"):
            e.append(f"engine.speculative.method {sp.method!r} needs trained speculator heads, which this engine "
                     "does not load; use 'draft' or 'ngram'")
        elif sp.method not in ("draft", "ngram"):
            e.append(f"engine.speculative.method must be draft|ngram, got {sp.method!r}")
        if sp.method == "ngram":
            if sp.draft_model or sp.draft_preset:
                e.append("engine.speculative: the ngram proposer takes no draft model")
            if not 1 <= sp.ngram_min <= sp.ngram_max <= 16:
                e.append("engine.speculative: need 1 <= ngram_min <= ngram_max <= 16")
    # fields kept for config-file parity whose non-default values this engine does not
    # implement: refused instead of silently ignored
    if m.expert_parallel_size not in (1, m.tensor_parallel_size):
        e.append("model.expert_parallel_size must be 1 or equal tensor_parallel_size (experts are split over "
                 "the tensor-parallel ranks)")
    if m.quantization is not None and m.quantization.group_size != 128:
        e.append(f"model.quantization.group_size must be 128 (the FP8 GEMM's block), got {m.quantization.group_size}")
    if g.kv_cache_dtype not in ("auto", m.dtype, "fp8", "fp8_e4m3", "fp8_e5m2"):
        e.append(f"engine.kv_cache_dtype must be auto (the model dtype), fp8, fp8_e4m3 or fp8_e5m2, "
                 f"got {g.kv_cache_dtype!r}")
    if not g.scheduling.enable_preemption:
        e.append("engine.scheduling.enable_preemption: false is not supported (a full KV cache preempts by "
                 "engine.scheduling.preemption_mode)")
    if g.scheduling.delay_factor != 0.0:
        e.append("engine.scheduling.delay_factor must be 0 (prompts are scheduled as soon as blocks allow)")
    if cfg.logging.level.lower() not in ("trace", "debug", "info", "warn", "warning", "error"):
        e.append(f"logging.level invalid: {cfg.logging.level!r}")
    if cfg.logging.format not in ("pretty", "compact", "json"):
        e.append("logging.format must be pretty|compact|json")
    pg = cfg.metrics.push_gateway
    if pg is not None:
        if not pg.url.startswith(("http://", "https://")):
            e.append(f"metrics.push_gateway.url must be an http(s) URL, got {pg.url!r}")
        if not pg.job:
            e.append("metrics.push_gateway.job must not be empty")
        if not pg.interval_seconds > 0:
            e.append(f"metrics.push_gateway.interval_seconds must be > 0, got {pg.interval_seconds}")
    return e


def validate_config(cfg) -> None:
    errs = collect_errors(cfg)
    if errs:
        raise ConfigError("invalid configuration:\n  - " + "\n  - ".join(errs))
