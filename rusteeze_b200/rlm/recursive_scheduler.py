"""Call tree for recursive sub-calls.

Semantics from crates/rusteeze-engine/src/recursive_scheduler.rs: spawning
children with depth and pending limits (:57-195), batch spawn, priority
`decay ** depth` (:234-260), ready calls scheduled with per-level
concurrency (16 by default, :347-471), per-call timeouts (120 s, :372-390),
completion, failure with cascading cancellation of descendants
(:474-553), and cancellation.  The reference builds this tree but its
engine never consults it (recursive_engine.rs:283); here the RLM engine
submits every sub-call through it, so limits and cancellation are real.
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional


class CallState(str, enum.Enum):
    PENDING = "pending"
    RUNNING = "running"
    DONE = "done"
    FAILED = "failed"
    CANCELLED = "cancelled"
    TIMED_OUT = "timed_out"


@dataclass
class SchedulerLimits:
    max_depth: int = 3
    max_pending: int = 1000
    per_level_concurrency: int = 16
    call_timeout_s: float = 120.0
    priority_decay: float = 0.8


@dataclass
class CallNode:
    call_id: int
    parent: Optional[int]
    depth: int
    prompt: str
    instruction: str
    priority: float
    state: CallState = CallState.PENDING
    children: List[int] = field(default_factory=list)
    result: Optional[str] = None
    error: Optional[str] = None
    started: Optional[float] = None
    finished: Optional[float] = None


_TERMINAL = (CallState.DONE, CallState.FAILED, CallState.CANCELLED, CallState.TIMED_OUT)
_DEAD = (CallState.FAILED, CallState.CANCELLED, CallState.TIMED_OUT)


class RecursiveScheduler:
    def __init__(self, limits: Optional[SchedulerLimits] = None):
        self.limits = limits or SchedulerLimits()
        self.nodes: Dict[int, CallNode] = {}
        self._ids = itertools.count(1)
        root = CallNode(0, None, 0, "", "", 1.0, CallState.RUNNING, started=time.monotonic())
        self.nodes[0] = root

    # ------------------------------------------------------------------ spawn
    def spawn(self, parent: int, prompt: str, instruction: str) -> int:
        p = self.nodes[parent]
        depth = p.depth + 1
        if depth > self.limits.max_depth:
            raise RecursionError(f"max recursion depth {self.limits.max_depth} exceeded")
        if self.num_pending() >= self.limits.max_pending:
            raise RuntimeError(f"too many pending sub-calls ({self.limits.max_pending})")
        cid = next(self._ids)
        node = CallNode(cid, parent, depth, prompt, instruction, self.limits.priority_decay ** depth)
        if self._under_dead(parent):
            # a call on the path to the root already failed, was cancelled or timed out (its
            # model output can still arrive and ask for sub-calls): born cancelled, never run
            node.state = CallState.CANCELLED
            node.finished = time.monotonic()
        self.nodes[cid] = node
        p.children.append(cid)
        return cid

    def _under_dead(self, cid: Optional[int]) -> bool:
        while cid is not None:
            n = self.nodes[cid]
            if n.state in _DEAD:
                return True
            cid = n.parent
        return False

    def spawn_batch(self, parent: int, items: List[tuple]) -> List[int]:
        return [self.spawn(parent, pr, ins) for pr, ins in items]

    # ------------------------------------------------------------------ scheduling
    def num_pending(self) -> int:
        return sum(1 for n in self.nodes.values() if n.state == CallState.PENDING)

    def ready(self) -> List[CallNode]:
        """Pending calls to start now: highest priority first, at most
        per_level_concurrency running per depth level."""
        running: Dict[int, int] = {}
        for n in self.nodes.values():
            if n.state == CallState.RUNNING:
                running[n.depth] = running.get(n.depth, 0) + 1
        out = []
        for n in sorted((n for n in self.nodes.values() if n.state == CallState.PENDING),
                        key=lambda n: (-n.priority, n.call_id)):
            if running.get(n.depth, 0) < self.limits.per_level_concurrency:
                running[n.depth] = running.get(n.depth, 0) + 1
                out.append(n)
        return out

    def start(self, cid: int) -> None:
        n = self.nodes[cid]
        if n.state != CallState.PENDING:
            return                     # only pending calls start (a cancelled one stays cancelled)
        n.state = CallState.RUNNING
        n.started = time.monotonic()

    def complete(self, cid: int, result: str) -> None:
        n = self.nodes[cid]
        if n.state in _TERMINAL:
            return                     # terminal states are final
        n.state = CallState.DONE
        n.result = result
        n.finished = time.monotonic()

    def fail(self, cid: int, error: str) -> None:
        n = self.nodes[cid]
        if n.state in _TERMINAL:
            return
        n.state = CallState.FAILED
        n.error = error
        n.finished = time.monotonic()
        for c in list(n.children):
            self.cancel(c)

    def cancel(self, cid: int) -> None:
        """Cancels a call and everything still pending or running below it; calls that
        already ended keep their state, but the cascade goes through them (a finished
        call can have sub-calls still queued)."""
        n = self.nodes[cid]
        if n.state not in _TERMINAL:
            n.state = CallState.CANCELLED
            n.finished = time.monotonic()
        for c in list(n.children):
            self.cancel(c)

    def check_timeouts(self, now: Optional[float] = None) -> List[int]:
        now = time.monotonic() if now is None else now
        out = []
        for n in self.nodes.values():
            if n.state == CallState.RUNNING and n.call_id != 0 and n.started is not None and \
                    now - n.started > self.limits.call_timeout_s:
                n.state = CallState.TIMED_OUT
                n.finished = now
                for c in list(n.children):
                    self.cancel(c)
                out.append(n.call_id)
        return out

    def stats(self) -> Dict[str, int]:
        d: Dict[str, int] = {}
        for n in self.nodes.values():
            d[n.state.value] = d.get(n.state.value, 0) + 1
        d["max_depth"] = max(n.depth for n in self.nodes.values())
        return d
