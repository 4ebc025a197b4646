"""Data-parallel replica router.

Counterpart of crates/rusteeze-engine/src/router.rs (least-loaded /
round-robin / random selection over N backends, manual health flags, a
log2 latency histogram with p50/p99; :13-274), which nothing in the
reference calls.  Here a `ReplicaRouter` fronts several engine replicas
(8 x TP1 on one box, one GPU each) for the data-parallel serving front end
(`engine.dp_engine.ReplicatedAsyncEngine`); health is driven by a prober
callback (the replica engine's readiness).

`prefix_affinity` (not in the reference) sends requests whose prompts start alike to the
same replica, so its prefix cache serves the shared part: the key is a hash of the
prompt's first `AFFINITY_TOKENS` tokens, and the replica is chosen by rendezvous hashing
(the live replica with the highest hash of (key, name)), so a replica that goes down or
comes back moves only its own keys.  A load guard sends the request to the least-loaded
replica instead when the chosen one has `AFFINITY_SLACK` more requests in flight.
"""
from __future__ import annotations

import enum
import hashlib
import math
import random
import threading
from dataclasses import dataclass, field
from typing import Callable, List, Optional


class Policy(str, enum.Enum):
    LEAST_LOADED = "least_loaded"
    ROUND_ROBIN = "round_robin"
    RANDOM = "random"
    PREFIX_AFFINITY = "prefix_affinity"


AFFINITY_TOKENS = 256
AFFINITY_SLACK = 8


def affinity_key(prompt_token_ids=None, prompt: str = None) -> int:
    """A stable key of a prompt's opening: its first AFFINITY_TOKENS token ids, or (text
    prompts, before tokenisation) its first 4 * AFFINITY_TOKENS characters."""
    if prompt_token_ids is not None:
        data = b",".join(str(int(t)).encode() for t in list(prompt_token_ids)[:AFFINITY_TOKENS])
    else:
        data = (prompt or "")[:4 * AFFINITY_TOKENS].encode("utf-8", "surrogatepass")
    return int.from_bytes(hashlib.blake2b(data, digest_size=8).digest(), "little")


def _rendezvous(key: int, name: str) -> int:
    return int.from_bytes(hashlib.blake2b(f"{key}:{name}".encode(), digest_size=8).digest(), "little")


class LatencyHistogram:
    """log2-bucketed latency histogram in microseconds (bucket i: [2^i, 2^(i+1)) us)."""

    def __init__(self, buckets: int = 40):
        self.counts = [0] * buckets
        self.n = 0

    def record(self, seconds: float) -> None:
        us = max(1.0, seconds * 1e6)
        i = min(len(self.counts) - 1, int(math.log2(us)))
        self.counts[i] += 1
        self.n += 1

    def percentile(self, q: float) -> Optional[float]:
        if self.n == 0:
            return None
        target = max(1, math.ceil(q / 100.0 * self.n))     # rank of the q-th percentile sample
        c = 0
        for i, k in enumerate(self.counts):
            c += k
            if c >= target:
                return (2 ** i) * 1.5 / 1e6   # bucket midpoint, seconds
        return None


@dataclass
class Replica:
    name: str
    backend: object
    healthy: bool = True
    in_flight: int = 0
    served: int = 0
    errors: int = 0
    latency: LatencyHistogram = field(default_factory=LatencyHistogram)


class ReplicaRouter:
    def __init__(self, replicas: List[Replica], policy: Policy = Policy.LEAST_LOADED, seed: int = 0,
                 prober: Optional[Callable[[Replica], bool]] = None):
        if not replicas:
            raise ValueError("router needs at least one replica")
        self.replicas = replicas
        self.policy = Policy(policy)
        self._rr = 0
        self._rng = random.Random(seed)
        self._lock = threading.Lock()
        self.prober = prober

    def probe(self) -> None:
        if self.prober is None:
            return
        for r in self.replicas:
            try:
                r.healthy = bool(self.prober(r))
            except Exception:  # noqa: BLE001 -- a failing probe marks the replica down
                r.healthy = False

    def set_health(self, name: str, healthy: bool) -> None:
        for r in self.replicas:
            if r.name == name:
                r.healthy = healthy
                return
        raise KeyError(f"no replica named {name!r}")

    def select(self, key: Optional[int] = None) -> Replica:
        """Picks a live replica; `key` (an `affinity_key`) is used by `prefix_affinity`."""
        with self._lock:
            live = [r for r in self.replicas if r.healthy]
            if not live:
                raise RuntimeError("no healthy replica")
            if self.policy == Policy.PREFIX_AFFINITY and key is not None:
                r = max(live, key=lambda x: _rendezvous(key, x.name))
                least = min(live, key=lambda x: (x.in_flight, x.served))
                if r.in_flight - least.in_flight >= AFFINITY_SLACK:
                    r = least
            elif self.policy == Policy.ROUND_ROBIN:
                r = live[self._rr % len(live)]
                self._rr += 1
            elif self.policy == Policy.RANDOM:
                r = self._rng.choice(live)
            else:
                r = min(live, key=lambda x: (x.in_flight, x.served))
            r.in_flight += 1
            return r

    def release(self, r: Replica, latency_s: Optional[float] = None, error: bool = False) -> None:
        with self._lock:
            r.in_flight = max(0, r.in_flight - 1)
            r.served += 1
            if error:
                r.errors += 1
            if latency_s is not None:
                r.latency.record(latency_s)

    def stats(self) -> List[dict]:
        return [{"name": r.name, "healthy": r.healthy, "in_flight": r.in_flight, "served": r.served,
                 "errors": r.errors, "p50_s": r.latency.percentile(50), "p99_s": r.latency.percentile(99)}
                for r in self.replicas]
