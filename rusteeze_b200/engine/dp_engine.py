"""Data-parallel serving: several engine replicas behind one HTTP front end.

The reference carries a replica router (crates/rusteeze-engine/src/router.rs:13-274:
least-loaded / round-robin / random over N backends, health flags, latency
histogram) that its server never calls.  Here `model.data_parallel_size = D > 1`
makes `serve()` build D `LLMEngine` replicas -- replica i owns GPU cuda:i (or
the CPU) with its own weights, KV cache, CUDA graphs and engine thread -- and
this front end, which the HTTP app uses exactly like a single `AsyncLLMEngine`:

  * every request goes to the replica `ReplicaRouter` picks (least-loaded by
    default); health is each replica's readiness, so a replica whose step
    raised or stalled stops receiving requests while the others keep serving;
  * aborts go to the replica that owns the request;
  * `stats()` sums the replicas' counters and reports per-replica router state;
  * step observers (the Prometheus metrics) are called with a view that sums
    the replicas' queues and KV blocks, serialised by a lock because every
    replica steps on its own thread.

Replicas share nothing on the device, so requests never cross NVLink; the
engine threads hold the GIL only for host-side scheduling between launches.
"""
from __future__ import annotations

import asyncio
import copy
import threading
import time
from typing import AsyncIterator, Callable, Dict, List, Optional

from rusteeze_b200.core.errors import ServiceUnavailableError
from rusteeze_b200.core.outputs import RequestOutput
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.router import Policy, Replica, ReplicaRouter, affinity_key


def replica_configs(config) -> List:
    """One config per replica: replica i runs on cuda:i (or the CPU), TP 1, DP 1."""
    import torch
    d = config.model.data_parallel_size
    dev = config.model.device
    if dev == "auto":
        dev = "cuda" if torch.cuda.is_available() else "cpu"
    if dev.startswith("cuda") and d > torch.cuda.device_count():
        raise ValueError(f"data_parallel_size {d} needs {d} GPUs; {torch.cuda.device_count()} visible")
    out = []
    for i in range(d):
        c = copy.deepcopy(config)
        c.model.data_parallel_size = 1
        c.model.tensor_parallel_size = 1
        c.model.device = f"cuda:{i}" if dev.startswith("cuda") else dev
        out.append(c)
    return out


class _SummedScheduler:
    def __init__(self, engines):
        self._e = engines

    def __getattr__(self, name):        # num_waiting / num_running / num_swapped / num_preemptions
        return sum(getattr(e.scheduler, name) for e in self._e)


class _SummedBlocks:
    def __init__(self, engines):
        self._e = engines

    @property
    def num_gpu_blocks(self) -> int:
        return sum(e.bm.num_gpu_blocks for e in self._e)

    def num_free_gpu_blocks(self) -> int:
        return sum(e.bm.num_free_gpu_blocks() for e in self._e)

    def gpu_usage(self) -> float:
        total = self.num_gpu_blocks
        return 0.0 if total == 0 else 1.0 - self.num_free_gpu_blocks() / total

    def stats(self) -> dict:
        out: Dict[str, float] = {}
        for e in self._e:
            for k, v in e.bm.stats().items():
                if isinstance(v, (int, float)) and not isinstance(v, bool):
                    out[k] = out.get(k, 0) + v
        return out


class _SummedRequests:
    def __init__(self, engines):
        self._e = engines

    def __len__(self) -> int:
        return sum(len(e.requests) for e in self._e)


class ReplicaView:
    """What the HTTP app and the step observers see as "the engine": the model's
    identity from replica 0, queue and block counts summed over all replicas."""

    def __init__(self, front: "ReplicatedAsyncEngine"):
        self._front = front
        engines = [r.backend.engine for r in front.router.replicas]
        first = engines[0]
        self.tokenizer = first.tokenizer
        self.model_config = first.model_config
        self.eos_ids = first.eos_ids
        self.model_name = first.model_name
        self.max_model_len = first.max_model_len
        self.config = first.config
        self.scheduler = _SummedScheduler(engines)
        self.bm = _SummedBlocks(engines)
        self.requests = _SummedRequests(engines)
        self.observers = _FanOutObservers(self, engines)

    def stats(self) -> dict:
        return self._front.stats()


class _FanOutObservers:
    """`observers` list of the view: appending registers the observer on every replica,
    called with the summed view under one lock."""

    def __init__(self, view: ReplicaView, engines):
        self._view = view
        self._engines = engines
        self._fns: List[Callable] = []
        self._lock = threading.Lock()

    def __contains__(self, fn) -> bool:
        return fn in self._fns

    def __iter__(self):
        return iter(list(self._fns))

    def __len__(self) -> int:
        return len(self._fns)

    def append(self, fn: Callable) -> None:
        self._fns.append(fn)
        view, lock = self._view, self._lock

        def relay(_engine, so, dt, _fn=fn):
            with lock:
                _fn(view, so, dt)
        for e in self._engines:
            e.observers.append(relay)


class ReplicatedAsyncEngine:
    """Front end over D `AsyncLLMEngine` replicas with the single-engine client API
    (`generate`, `abort`, `stats`, `is_ready`, `engine`, `start`, `shutdown`)."""

    def __init__(self, replicas: List, policy: Policy = Policy.LEAST_LOADED, seed: int = 0):
        if not replicas:
            raise ValueError("data-parallel front end needs at least one replica")
        self.router = ReplicaRouter([Replica(f"dp{i}", ae) for i, ae in enumerate(replicas)], Policy(policy),
                                    seed=seed, prober=lambda r: r.backend.is_ready)
        self._owner: Dict[str, Replica] = {}
        self.engine = ReplicaView(self)

    @classmethod
    def from_config(cls, config, request_timeout_s: Optional[float] = None) -> "ReplicatedAsyncEngine":
        from rusteeze_b200.engine.async_engine import AsyncLLMEngine
        from rusteeze_b200.engine.llm_engine import LLMEngine
        t = request_timeout_s or config.engine.request_timeout_seconds
        reps = [AsyncLLMEngine(LLMEngine(c), request_timeout_s=t) for c in replica_configs(config)]
        return cls(reps, Policy(config.server.router_policy), seed=config.model.seed)

    @property
    def replicas(self) -> List:
        return [r.backend for r in self.router.replicas]

    # ------------------------------------------------------------------ lifecycle
    def start(self) -> "ReplicatedAsyncEngine":
        for ae in self.replicas:
            ae.start()
        return self

    def shutdown(self, timeout: float = 10.0) -> None:
        for ae in self.replicas:
            ae.shutdown(timeout)

    @property
    def is_ready(self) -> bool:
        return any(ae.is_ready for ae in self.replicas)

    # ------------------------------------------------------------------ client API
    async def generate(self, prompt: Optional[str], params: SamplingParams, request_id: str,
                       prompt_token_ids: Optional[List[int]] = None,
                       priority: int = 0) -> AsyncIterator[RequestOutput]:
        self.router.probe()
        key = (affinity_key(prompt_token_ids, prompt) if self.router.policy == Policy.PREFIX_AFFINITY else None)
        try:
            rep = self.router.select(key)
        except RuntimeError as e:
            raise ServiceUnavailableError(f"no ready replica: {e}") from None
        self._owner[request_id] = rep
        t0 = time.monotonic()
        failed = False
        agen = rep.backend.generate(prompt, params, request_id, prompt_token_ids, priority)
        try:
            async for out in agen:
                yield out
        except (GeneratorExit, asyncio.CancelledError):
            raise                        # the client went away: not the replica's fault
        except BaseException:
            failed = True
            raise
        finally:
            await agen.aclose()
            self._owner.pop(request_id, None)
            self.router.release(rep, time.monotonic() - t0, error=failed)

    async def embed(self, inputs, pooling: str = "last", normalize: bool = True) -> list:
        """Embeddings on the replica the router picks."""
        self.router.probe()
        try:
            rep = self.router.select()
        except RuntimeError as e:
            raise ServiceUnavailableError(f"no ready replica: {e}") from None
        t0 = time.monotonic()
        failed = False
        try:
            return await rep.backend.embed(inputs, pooling, normalize)
        except BaseException:
            failed = True
            raise
        finally:
            self.router.release(rep, time.monotonic() - t0, error=failed)

    def abort(self, request_id: str) -> None:
        rep = self._owner.get(request_id)
        for r in ([rep] if rep is not None else self.router.replicas):
            r.backend.abort(request_id)

    def stats(self) -> dict:
        per = [ae.stats() for ae in self.replicas]
        out: Dict[str, object] = {}
        for d in per:
            for k, v in d.items():
                if isinstance(v, (int, float)) and not isinstance(v, bool):
                    out[k] = out.get(k, 0) + v
        blocks = sum(d.get("num_gpu_blocks", 0) for d in per)
        out["kv_cache_usage"] = (sum(d.get("kv_cache_usage", 0.0) * d.get("num_gpu_blocks", 0) for d in per)
                                 / blocks) if blocks else 0.0
        out["uptime_s"] = max(d.get("uptime_s", 0.0) for d in per)
        out["healthy"] = self.is_ready
        out["data_parallel_size"] = len(per)
        out["replicas"] = self.router.stats()
        return out
