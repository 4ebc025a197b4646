"""Config loading with precedence defaults < file < env < CLI overrides.

File format by extension (.yaml/.yml, .toml, .json) as in
crates/rusteeze-config/src/loader.rs:12-43; the RUSTEEZE_* environment
overrides are the same names as loader.rs:130-188; the default search path
list mirrors loader.rs:199-222.
"""
from __future__ import annotations

import json
import os
from typing import Any, Dict, Optional

from rusteeze_b200.config.config import Config, config_from_dict, merge_dict
from rusteeze_b200.config.validation import validate_config
from rusteeze_b200.core.errors import ConfigError

DEFAULT_SEARCH_PATHS = [
    "rusteeze.yaml", "rusteeze.yml", "rusteeze.toml", "rusteeze.json",
    "config/rusteeze.yaml", "config.yaml",
    os.path.expanduser("~/.config/rusteeze/config.yaml"),
    "/etc/rusteeze/config.yaml",
]

# env var suffix -> (section, key, type)
ENV_OVERRIDES = {
    "MODEL_PATH": ("model", "path", str),
    "MODEL": ("model", "path", str),
    "MODEL_NAME": ("model", "name", str),
    "MODEL_PRESET": ("model", "preset", str),
    "MODEL_DTYPE": ("model", "dtype", str),
    "MODEL_DEVICE": ("model", "device", str),
    "MODEL_MAX_LEN": ("model", "max_model_len", int),
    "TENSOR_PARALLEL": ("model", "tensor_parallel_size", int),
    "EXPERT_PARALLEL": ("model", "expert_parallel_size", int),
    "HOST": ("server", "host", str),
    "PORT": ("server", "port", int),
    "API_KEY": ("server", "api_key", str),
    "MAX_SEQS": ("engine", "max_num_seqs", int),
    "MAX_TOKENS": ("engine", "max_num_batched_tokens", int),
    "GPU_MEMORY_UTIL": ("engine", "gpu_memory_utilization", float),
    "COMM_BACKEND": ("engine", "comm_backend", str),
    "LOG_LEVEL": ("logging", "level", str),
}


def detect_format(path: str) -> str:
    ext = os.path.splitext(path)[1].lower()
    if ext in (".yaml", ".yml"):
        return "yaml"
    if ext == ".toml":
        return "toml"
    if ext == ".json":
        return "json"
    raise ConfigError(f"unsupported config file extension {ext!r} (use .yaml/.yml/.toml/.json)")


def parse_text(text: str, fmt: str) -> Dict[str, Any]:
    if fmt not in ("yaml", "toml", "json"):
        raise ConfigError(f"unknown format {fmt}")
    try:
        if fmt == "yaml":
            import yaml
            d = yaml.safe_load(text) or {}
        elif fmt == "toml":
            import tomllib
            d = tomllib.loads(text)
        else:
            d = json.loads(text)
    except Exception as e:  # noqa: BLE001 -- yaml / toml / json parse errors
        raise ConfigError(f"cannot parse the {fmt} config: {e}") from None
    if not isinstance(d, dict):
        raise ConfigError(f"a {fmt} config must be a mapping of sections, got {type(d).__name__}")
    return d


def load_file(path: str) -> Dict[str, Any]:
    if not os.path.exists(path):
        raise ConfigError(f"config file not found: {path}")
    with open(path) as f:
        return parse_text(f.read(), detect_format(path))


def env_overrides(prefix: str = "RUSTEEZE", environ=None) -> Dict[str, Any]:
    environ = os.environ if environ is None else environ
    out: Dict[str, Any] = {}
    for suffix, (sec, key, typ) in ENV_OVERRIDES.items():
        v = environ.get(f"{prefix}_{suffix}")
        if v is None:
            continue
        try:
            val = typ(v)
        except ValueError:
            raise ConfigError(f"{prefix}_{suffix}={v!r} is not a valid {typ.__name__}") from None
        out.setdefault(sec, {})[key] = val
    if "LOG_LEVEL" in environ and "logging" not in out:
        out.setdefault("logging", {})["level"] = environ["LOG_LEVEL"]
    return out


def find_default_config() -> Optional[str]:
    for p in DEFAULT_SEARCH_PATHS:
        if os.path.exists(p):
            return p
    return None


class ConfigLoader:
    def __init__(self, path: Optional[str] = None, env_prefix: str = "RUSTEEZE",
                 search_defaults: bool = False, environ=None):
        self.path = path
        self.env_prefix = env_prefix
        self.search_defaults = search_defaults
        self.environ = environ

    def load(self, cli_overrides: Optional[Dict[str, Any]] = None, validate: bool = True) -> Config:
        d: Dict[str, Any] = {}
        path = self.path or (os.environ.get(f"{self.env_prefix}_CONFIG") if self.environ is None
                             else self.environ.get(f"{self.env_prefix}_CONFIG"))
        if path is None and self.search_defaults:
            path = find_default_config()
        if path:
            d = merge_dict(d, load_file(path))
        d = merge_dict(d, env_overrides(self.env_prefix, self.environ))
        if cli_overrides:
            d = merge_dict(d, {s: {k: v for k, v in sec.items() if v is not None}
                               for s, sec in cli_overrides.items()})
        cfg = config_from_dict(d)
        if validate:
            validate_config(cfg)
        return cfg


def load_config(path: Optional[str] = None, cli_overrides=None, **kw) -> Config:
    return ConfigLoader(path, **kw).load(cli_overrides)
