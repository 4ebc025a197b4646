"""Host-side span tracing in the Chrome trace-event format (open the file in Perfetto or
chrome://tracing).

Enabled by `RUSTEEZE_TRACE=<path.json>` (or `enable(path)`): every `nvtx_range` of the
engine (schedule / launch / execute / finish phases, ...) and every `span()` records a
complete event {name, ph "X", ts, dur, pid, tid, args}; the file is written at exit or by
`dump()`.  This is the tracing counterpart of the reference's `tracing` subscriber
(crates/rusteeze-metrics/src/tracing_setup.rs:78-180) for a box without nsys or an
OpenTelemetry collector: spans are kept in memory (bounded by `max_events`) and cost a
`perf_counter_ns` pair each when enabled, nothing when not.
"""
from __future__ import annotations

import atexit
import json
import os
import threading
import time
from typing import Dict, List, Optional

_lock = threading.Lock()
_events: List[Dict] = []
_path: Optional[str] = None
_max_events = 1_000_000
_dropped = 0
_t0 = time.perf_counter_ns()


def enabled() -> bool:
    return _path is not None


def enable(path: str, max_events: int = 1_000_000) -> None:
    global _path, _max_events
    _path, _max_events = path, max_events


def disable() -> None:
    global _path
    _path = None


def record(name: str, t_start_ns: int, t_end_ns: int, args: Optional[Dict] = None) -> None:
    global _dropped
    if _path is None:
        return
    ev = {"name": name, "ph": "X", "ts": (t_start_ns - _t0) / 1e3, "dur": (t_end_ns - t_start_ns) / 1e3,
          "pid": os.getpid(), "tid": threading.get_ident() % (1 << 31)}
    if args:
        ev["args"] = args
    with _lock:
        if len(_events) < _max_events:
            _events.append(ev)
        else:
            _dropped += 1


class span:
    """`with span("name", key=value): ...` records one complete event when tracing is on."""

    __slots__ = ("name", "args", "t")

    def __init__(self, name: str, **args):
        self.name, self.args = name, args

    def __enter__(self):
        self.t = time.perf_counter_ns() if _path is not None else 0
        return self

    def __exit__(self, *exc):
        if self.t:
            record(self.name, self.t, time.perf_counter_ns(), self.args or None)
        return False


def dump(path: Optional[str] = None) -> Optional[str]:
    """Writes the recorded events (Chrome trace JSON) and returns the path."""
    path = path or _path
    if path is None:
        return None
    with _lock:
        data = {"traceEvents": list(_events), "displayTimeUnit": "ms",
                "otherData": {"dropped_events": _dropped, "producer": "rusteeze_b200"}}
    with open(path, "w") as f:
        json.dump(data, f)
    return path


def clear() -> None:
    global _dropped
    with _lock:
        _events.clear()
        _dropped = 0


if os.environ.get("RUSTEEZE_TRACE"):
    enable(os.environ["RUSTEEZE_TRACE"])
    atexit.register(dump)
