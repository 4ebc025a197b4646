"""Structured logging (pretty | compact | json) and optional OpenTelemetry.

Mirrors crates/rusteeze-metrics/src/tracing_setup.rs:79-225: level and
format from config or LOG_LEVEL / LOG_FORMAT, optional file output, OTLP
export when OTLP_ENABLED=1 and the opentelemetry SDK is importable (it is
not in this image, so the exporter is skipped with a warning).
"""
from __future__ import annotations

import json
import logging
import os
import sys
import time
from typing import Optional

_LEVELS = {"trace": logging.DEBUG, "debug": logging.DEBUG, "info": logging.INFO, "warn": logging.WARNING,
           "warning": logging.WARNING, "error": logging.ERROR}


class JsonFormatter(logging.Formatter):
    def format(self, rec: logging.LogRecord) -> str:
        d = {"ts": time.strftime("%Y-%m-%dT%H:%M:%S", time.gmtime(rec.created)) + f".{int(rec.msecs):03d}Z",
             "level": rec.levelname.lower(), "target": rec.name, "message": rec.getMessage()}
        for k in ("request_id", "rank", "step"):
            if hasattr(rec, k):
                d[k] = getattr(rec, k)
        if rec.exc_info:
            d["exception"] = self.formatException(rec.exc_info)
        return json.dumps(d)


def init_logging(level: Optional[str] = None, fmt: Optional[str] = None, file: Optional[str] = None,
                 service_name: str = "rusteeze") -> logging.Logger:
    level = (level or os.environ.get("LOG_LEVEL", "info")).lower()
    fmt = fmt or os.environ.get("LOG_FORMAT", "pretty")
    root = logging.getLogger("rusteeze")
    root.setLevel(_LEVELS.get(level, logging.INFO))
    for h in list(root.handlers):
        root.removeHandler(h)
    h: logging.Handler = logging.FileHandler(file) if file else logging.StreamHandler(sys.stderr)
    if fmt == "json":
        h.setFormatter(JsonFormatter())
    elif fmt == "compact":
        h.setFormatter(logging.Formatter("%(levelname).1s %(name)s: %(message)s"))
    else:
        h.setFormatter(logging.Formatter("%(asctime)s %(levelname)-5s %(name)s: %(message)s"))
    root.addHandler(h)
    root.propagate = False
    if os.environ.get("OTLP_ENABLED", "0") in ("1", "true"):
        try:
            import opentelemetry  # noqa: F401
            root.info("OTLP export enabled (endpoint %s)", os.environ.get("OTLP_ENDPOINT", "localhost:4317"))
        except ImportError:
            root.warning("OTLP_ENABLED set but the opentelemetry SDK is not installed; tracing export skipped")
    return root


class nvtx_range:
    """NVTX range around an engine phase (no-op when CUDA/NVTX is unavailable); with host
    tracing on (`RUSTEEZE_TRACE`, metrics/trace.py) it also records a trace span."""

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        from rusteeze_b200.metrics import trace
        self.t = time.perf_counter_ns() if trace.enabled() else 0
        try:
            import torch
            if torch.cuda.is_available():
                torch.cuda.nvtx.range_push(self.name)
                self.on = True
                return self
        except Exception:  # noqa: BLE001
            pass
        self.on = False
        return self

    def __exit__(self, *exc):
        if self.on:
            import torch
            torch.cuda.nvtx.range_pop()
        if self.t:
            from rusteeze_b200.metrics import trace
            trace.record(self.name, self.t, time.perf_counter_ns())
        return False
