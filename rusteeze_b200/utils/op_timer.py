"""Per-op device time of engine steps, from CUDA events on the launching stream.

`OP_TIMER.section(name)` brackets a group of kernel launches (a GEMM with its fused
collective, the attention, the norm + all-gather, ...) with two CUDA events when the
timer is enabled; `report()` waits for them and returns milliseconds per section.
Enabled only for measurement runs (`bench.py --op-split`): each section costs two event
records, and inside a CUDA-graph capture it times nothing (the replay of a captured
decode step is timed as one `decode_graph` section by the runner).  Sections are
device time between the two records on one stream, so they include waits on peers
inside fused collectives: at N GPUs they show where the step waits, which is what
limits the scaling.
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import torch


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NULL = _Null()


class _Section:
    __slots__ = ("t", "name", "e0")

    def __init__(self, t: "OpTimer", name: str):
        self.t, self.name = t, name

    def __enter__(self):
        self.e0 = self.t._event()
        self.e0.record()
        return self

    def __exit__(self, *exc):
        e1 = self.t._event()
        e1.record()
        self.t.pending.append((self.name, self.e0, e1))
        return False


class OpTimer:
    def __init__(self):
        self.enabled = False
        self.pending: List[Tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self.totals: Dict[str, float] = {}
        self.counts: Dict[str, int] = {}
        self._free: List[torch.cuda.Event] = []

    def _event(self) -> torch.cuda.Event:
        return self._free.pop() if self._free else torch.cuda.Event(enable_timing=True)

    def section(self, name: str):
        if not self.enabled or not torch.cuda.is_available() or torch.cuda.is_current_stream_capturing():
            return _NULL
        return _Section(self, name)

    def start(self) -> None:
        self.pending.clear()
        self.totals.clear()
        self.counts.clear()
        self.enabled = True

    def stop(self) -> None:
        self.enabled = False

    def report(self) -> Dict[str, float]:
        """Milliseconds per section name, summed over the window (synchronises)."""
        if self.pending:
            torch.cuda.synchronize()
        for name, e0, e1 in self.pending:
            self.totals[name] = self.totals.get(name, 0.0) + e0.elapsed_time(e1)
            self.counts[name] = self.counts.get(name, 0) + 1
            self._free += (e0, e1)
        self.pending.clear()
        return dict(self.totals)


OP_TIMER = OpTimer()

# every section name the engine uses, in a fixed order (ranks all-reduce a vector of these)
SECTIONS = ["embed", "qkv_gemm", "rope_kv", "attention", "o_gemm_rs", "norm_ag", "gate_up_gemm",
            "down_gemm_rs", "moe", "final_norm", "lm_head", "decode_graph", "sample"]
