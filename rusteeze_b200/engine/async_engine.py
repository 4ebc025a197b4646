"""Asynchronous front end over LLMEngine for the HTTP server.

The reference's `Engine::generate` runs a single step per request and waits
on a oneshot channel (crates/rusteeze-engine/src/engine.rs:239-300);
`generate_stream` relies on an `Engine::run` loop nobody spawns
(engine.rs:303-354, 558-572).  Here one dedicated thread owns the engine and
runs `step()` back to back while work exists; requests and aborts arrive
through a thread-safe inbox; every RequestOutput is pushed to the asyncio
queue of its request with `call_soon_threadsafe`, so HTTP handlers stream
tokens as they are produced.  Request timeouts (engine.rs:295, default
600 s) abort the request inside the engine.  A watchdog marks the engine
unhealthy when a step raises or stalls longer than `stall_timeout_s`
(`/health/ready` then reports 503).
"""
from __future__ import annotations

import asyncio
import logging
import queue
import threading
import time
import traceback
from dataclasses import dataclass
from typing import AsyncIterator, Dict, List, Optional

from rusteeze_b200.core.errors import DistributedError, RequestTimeoutError, ServiceUnavailableError
from rusteeze_b200.core.outputs import RequestOutput
from rusteeze_b200.core.sampling_params import SamplingParams

log = logging.getLogger("rusteeze.async_engine")


def _settle(fut: "asyncio.Future", result, error) -> None:
    if fut.done():                     # the caller gave up
        return
    if error is not None:
        fut.set_exception(error)
    else:
        fut.set_result(result)


@dataclass
class _Submit:
    request_id: str
    prompt: Optional[str]
    prompt_token_ids: Optional[List[int]]
    params: SamplingParams
    priority: int
    loop: asyncio.AbstractEventLoop
    q: asyncio.Queue


class AsyncLLMEngine:
    def __init__(self, engine, request_timeout_s: float = 600.0, stall_timeout_s: float = 120.0,
                 max_worker_recoveries: int = 3):
        self.engine = engine
        self.max_worker_recoveries = max_worker_recoveries
        self.recovering = False
        self.request_timeout_s = request_timeout_s
        self.stall_timeout_s = stall_timeout_s
        self._inbox: "queue.Queue" = queue.Queue()
        self._streams: Dict[str, _Submit] = {}
        self._deadlines: Dict[str, float] = {}
        self._wake = threading.Event()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.healthy = True
        self.last_error: Optional[str] = None
        self.last_step_start: Optional[float] = None
        self.started_at = time.time()
        self.requests_processed = 0
        self._last_status_check = 0.0

    # ------------------------------------------------------------------ lifecycle
    def start(self) -> "AsyncLLMEngine":
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, name="rusteeze-engine", daemon=True)
            self._thread.start()
        return self

    def shutdown(self, timeout: float = 10.0) -> None:
        self._stop.set()
        self._wake.set()
        if self._thread is not None:
            self._thread.join(timeout)

    @property
    def is_ready(self) -> bool:
        if not self.healthy or self.recovering or self._thread is None or not self._thread.is_alive():
            return False
        t = self.last_step_start
        return t is None or time.monotonic() - t < self.stall_timeout_s

    # ------------------------------------------------------------------ client API
    async def generate(self, prompt: Optional[str], params: SamplingParams, request_id: str,
                       prompt_token_ids: Optional[List[int]] = None,
                       priority: int = 0) -> AsyncIterator[RequestOutput]:
        if not self.is_ready:
            raise ServiceUnavailableError(self.last_error or "engine is not ready")
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        self._inbox.put(("add", _Submit(request_id, prompt, prompt_token_ids, params, priority, loop, q)))
        self._wake.set()
        try:
            while True:
                item = await q.get()
                if isinstance(item, BaseException):
                    raise item
                yield item
                if item.finished:
                    return
        finally:
            # client went away or finished: make sure the engine drops it
            self._inbox.put(("abort", request_id))
            self._wake.set()

    def abort(self, request_id: str) -> None:
        self._inbox.put(("abort", request_id))
        self._wake.set()

    async def embed(self, inputs: List[List[int]], pooling: str = "last", normalize: bool = True) -> list:
        """Embeddings (`LLMEngine.embed`), computed on the engine thread between steps."""
        if not self.is_ready:
            raise ServiceUnavailableError(self.last_error or "engine is not ready")
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self._inbox.put(("embed", (inputs, pooling, normalize, loop, fut)))
        self._wake.set()
        return await fut

    def stats(self) -> dict:
        d = dict(self.engine.stats())
        d["uptime_s"] = time.time() - self.started_at
        d["requests_processed"] = self.requests_processed
        d["healthy"] = self.healthy
        return d

    # ------------------------------------------------------------------ engine thread
    @staticmethod
    def _push(sub: _Submit, item) -> bool:
        """Hands an item to the request's asyncio queue; False when the client's event loop
        is gone (its stream is then dropped), so one vanished client cannot stop the
        engine thread."""
        try:
            sub.loop.call_soon_threadsafe(sub.q.put_nowait, item)
            return True
        except RuntimeError:            # event loop closed
            return False

    def _drain_inbox(self) -> None:
        while True:
            try:
                kind, item = self._inbox.get_nowait()
            except queue.Empty:
                return
            if kind == "add":
                try:
                    self.engine.add_request(item.request_id, item.prompt, item.params, item.prompt_token_ids,
                                            priority=item.priority)
                    self._streams[item.request_id] = item
                    self._deadlines[item.request_id] = time.monotonic() + self.request_timeout_s
                except BaseException as e:  # noqa: BLE001 -- delivered to the caller
                    self._push(item, e)
            elif kind == "embed":
                inputs, pooling, normalize, loop, fut = item
                try:
                    if getattr(self.engine, "_inflight", None):
                        self._deliver(self.engine._drain_inflight())
                    res, err = self.engine.embed(inputs, pooling, normalize), None
                except BaseException as e:  # noqa: BLE001 -- delivered to the caller
                    res, err = None, e
                try:
                    loop.call_soon_threadsafe(_settle, fut, res, err)
                except RuntimeError:        # the caller's event loop is gone
                    pass
            elif kind == "abort":
                sub = self._streams.pop(item, None)
                if sub is not None:
                    req = self.engine.requests.get(item)
                    self.engine.abort_request(item)
                    self._deadlines.pop(item, None)
                    if req is not None:
                        # a caller still iterating the stream gets its final (aborted) output
                        self._push(sub, req.to_output(delta=True))

    def _expire(self) -> None:
        now = time.monotonic()
        for rid, dl in list(self._deadlines.items()):
            if now > dl:
                sub = self._streams.pop(rid, None)
                self._deadlines.pop(rid, None)
                self.engine.abort_request(rid)
                if sub is not None:
                    self._push(sub, RequestTimeoutError(f"request {rid} timed out"))

    def _check_device_status(self) -> None:
        """Kernels report protocol errors (an expired bounded wait, a corrupt
        block table) in a device status word instead of trapping; poll it about
        once per second and mark the engine unhealthy when it is set."""
        now = time.monotonic()
        if now - self._last_status_check < 1.0:
            return
        self._last_status_check = now
        dev = getattr(self.engine, "device", "cpu")
        if not str(dev).startswith("cuda"):
            return
        try:
            from rusteeze_b200 import ops
            code = int(ops.cuda_ext().status()[0])
        except Exception:  # noqa: BLE001
            return
        if code != 0:
            self.healthy = False
            self.last_error = f"device kernel status {code}"
            log.error("device kernel reported status %d; engine marked unhealthy", code)

    def _fail(self, e: BaseException) -> None:
        self.healthy = False
        self.last_error = f"engine step failed: {e!r}"
        log.error("engine step failed:\n%s", traceback.format_exc())
        for sub in self._streams.values():
            self._push(sub, ServiceUnavailableError(self.last_error))
        self._streams.clear()

    def _recover(self, launcher, err: BaseException) -> bool:
        """Worker-group recovery; returns False (engine unhealthy) when it fails too or when
        the engine has already been recovered `max_worker_recoveries` times."""
        if launcher.recoveries >= self.max_worker_recoveries:
            return False
        log.error("engine step failed with %r; replacing the tensor-parallel worker group", err)
        self.recovering = True            # /health/ready answers 503 meanwhile
        try:
            launcher.recover()
        except BaseException:  # noqa: BLE001
            log.error("worker-group recovery failed:\n%s", traceback.format_exc())
            return False
        finally:
            self.recovering = False
        return True

    def _loop(self) -> None:
        dev = str(getattr(self.engine, "device", "cpu"))
        if dev.startswith("cuda"):
            import torch
            torch.cuda.set_device(torch.device(dev))   # the current device is per thread
        while not self._stop.is_set():
            self._drain_inbox()
            self._expire()
            self._check_device_status()
            if not self.engine.has_unfinished_requests():
                self._wake.wait(0.05)
                self._wake.clear()
                continue
            self.last_step_start = time.monotonic()
            try:
                outs = self.engine.step()
            except DistributedError as e:
                # a tensor-parallel worker died: replace the worker group and keep serving
                # (the engine re-queues its live sequences as recompute preemptions)
                launcher = getattr(self.engine, "tp_launcher", None)
                if launcher is not None and self._recover(launcher, e):
                    continue
                self._fail(e)
                return
            except BaseException as e:  # noqa: BLE001
                self._fail(e)
                return
            finally:
                self.last_step_start = None
            self._deliver(outs)

    def _deliver(self, outs) -> None:
        """Hands each output to its request's stream."""
        for o in outs:
            sub = self._streams.get(o.request_id)
            if sub is None:
                continue
            if not self._push(sub, o):
                # the client is gone: stop generating for it
                self._streams.pop(o.request_id, None)
                self._deadlines.pop(o.request_id, None)
                if not o.finished:
                    self.engine.abort_request(o.request_id)
                continue
            if o.finished:
                self._streams.pop(o.request_id, None)
                self._deadlines.pop(o.request_id, None)
                self.requests_processed += 1
