"""Prometheus metrics, updated from the engine loop every step.

The reference defines three overlapping metric sets -- the collector registry
`rusteeze_inference_*` (crates/rusteeze-metrics/src/collector.rs:93-336), the
global `rusteeze_*` counters/gauges/histograms (counters.rs:15-34,
gauges.rs:18-44, histograms.rs:25-45), and a hand-formatted `/metrics` in the
API (crates/rusteeze-api/src/routes.rs:79-119) -- and the engine updates none
of them.  Here a single registry carries those names and `EngineMetrics`
is attached to the engine as a step observer, so every value is live.
Bucket boundaries follow the collector: TTFT 10 ms .. 5 s, inter-token
latency 1 .. 250 ms.
"""
from __future__ import annotations

import time
from typing import Optional

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest

CONTENT_TYPE = "text/plain; version=0.0.4; charset=utf-8"

TTFT_BUCKETS = (0.01, 0.025, 0.05, 0.075, 0.1, 0.15, 0.2, 0.3, 0.5, 0.75, 1.0, 2.0, 5.0)
ITL_BUCKETS = (0.001, 0.005, 0.01, 0.02, 0.03, 0.05, 0.075, 0.1, 0.15, 0.2, 0.25)
LAT_BUCKETS = (0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 30.0, 60.0, 120.0, 300.0)
STEP_BUCKETS = (0.001, 0.002, 0.005, 0.01, 0.02, 0.03, 0.05, 0.1, 0.2, 0.5, 1.0)


class EngineMetrics:
    def __init__(self, registry: Optional[CollectorRegistry] = None, model_name: str = "model"):
        r = self.registry = registry or CollectorRegistry()
        self.model = model_name
        p = "rusteeze_inference_"
        # collector set
        self.requests_total = Counter(p + "requests_total", "Requests by final status", ["status"], registry=r)
        self.requests_active = Gauge(p + "requests_active", "Requests in flight", registry=r)
        self.request_latency = Histogram(p + "request_latency_seconds", "End-to-end request latency",
                                         buckets=LAT_BUCKETS, registry=r)
        self.prompt_tokens = Counter(p + "prompt_tokens_total", "Prompt tokens processed", registry=r)
        self.generation_tokens = Counter(p + "generation_tokens_total", "Tokens generated", registry=r)
        self.tokens_per_second = Gauge(p + "tokens_per_second", "Generation throughput (last step)", registry=r)
        self.ttft = Histogram(p + "time_to_first_token_seconds", "Time to first token", buckets=TTFT_BUCKETS,
                              registry=r)
        self.itl = Histogram(p + "inter_token_latency_seconds", "Mean time per output token per request",
                             buckets=ITL_BUCKETS, registry=r)
        self.batch_size = Histogram(p + "batch_size", "Sequences per step", buckets=(1, 2, 4, 8, 16, 32, 64,
                                                                                       128, 256, 512), registry=r)
        self.batch_tokens = Histogram(p + "batch_tokens", "Tokens per step",
                                      buckets=(1, 16, 64, 256, 512, 1024, 2048, 4096, 8192, 16384), registry=r)
        self.batches_total = Counter(p + "batches_total", "Engine steps", registry=r)
        self.step_seconds = Histogram(p + "step_seconds", "Engine step wall time", buckets=STEP_BUCKETS, registry=r)
        self.queue_waiting = Gauge(p + "queue_waiting", "Waiting sequences", registry=r)
        self.queue_running = Gauge(p + "queue_running", "Running sequences", registry=r)
        self.queue_swapped = Gauge(p + "queue_swapped", "Swapped sequences", registry=r)
        self.queue_wait_time = Histogram(p + "queue_wait_seconds", "Arrival to first schedule",
                                         buckets=LAT_BUCKETS, registry=r)
        self.gpu_memory = Gauge(p + "gpu_memory_bytes", "GPU memory allocated", ["device"], registry=r)
        self.kv_usage = Gauge(p + "kv_cache_usage_ratio", "Fraction of KV blocks in use", registry=r)
        self.block_usage = Gauge(p + "block_usage", "KV blocks in use", registry=r)
        self.errors = Counter(p + "errors_total", "Errors by type", ["type"], registry=r)
        self.temperature = Histogram(p + "sampling_temperature", "Requested temperature",
                                     buckets=(0.0, 0.1, 0.3, 0.5, 0.7, 1.0, 1.5, 2.0), registry=r)
        self.top_p = Histogram(p + "sampling_top_p", "Requested top_p", buckets=(0.1, 0.5, 0.8, 0.9, 0.95, 1.0),
                               registry=r)
        self.prefix_hits = Counter(p + "prefix_cache_hits_total", "Prefix-cache block hits", registry=r)
        self.prefix_misses = Counter(p + "prefix_cache_misses_total", "Prefix-cache block misses", registry=r)
        self.preemptions = Counter(p + "preemptions_total", "Sequences preempted", registry=r)
        self.spec_accepted = Counter(p + "spec_decode_accepted_tokens_total", "Accepted draft tokens", registry=r)
        self.spec_proposed = Counter(p + "spec_decode_proposed_tokens_total", "Proposed draft tokens", registry=r)
        self.kernel_seconds = Histogram(p + "device_step_seconds", "Device time per step (CUDA events)",
                                        buckets=STEP_BUCKETS, registry=r)
        # global rusteeze_* set
        self.g_requests = Counter("rusteeze_requests_total", "Requests", ["status", "model", "endpoint"], registry=r)
        self.g_tokens = Counter("rusteeze_tokens_total", "Tokens", ["type", "model"], registry=r)
        self.g_active = Gauge("rusteeze_active_requests", "Active requests", registry=r)
        self.g_queue = Gauge("rusteeze_queue_size", "Queue size", registry=r)
        self.g_memory = Gauge("rusteeze_memory_bytes", "Memory", ["type"], registry=r)
        self.g_latency = Histogram("rusteeze_request_latency_seconds", "Request latency", ["endpoint"],
                                   buckets=LAT_BUCKETS, registry=r)
        self.g_token_latency = Histogram("rusteeze_token_latency_seconds", "Per-token latency",
                                         buckets=ITL_BUCKETS, registry=r)
        self.uptime = Gauge("rusteeze_uptime_seconds", "Process uptime", registry=r)
        self._t0 = time.time()
        self._last_prefix = (0, 0)
        self._last_preempt = 0

    # ------------------------------------------------------------------ engine observer
    def on_step(self, engine, sched_out, step_s: float) -> None:
        n_seq = len(sched_out.decodes) + len(sched_out.prefills)
        self.batches_total.inc()
        self.batch_size.observe(n_seq)
        self.batch_tokens.observe(sched_out.num_batched_tokens)
        self.step_seconds.observe(step_s)
        gen = sum(1 for s in sched_out.scheduled if s.sample)
        prompt = sum(s.num_new for s in sched_out.prefills)
        self.generation_tokens.inc(gen)
        self.prompt_tokens.inc(prompt)
        self.g_tokens.labels("generation", self.model).inc(gen)
        self.g_tokens.labels("prompt", self.model).inc(prompt)
        if step_s > 0:
            self.tokens_per_second.set(gen / step_s)
        sch = engine.scheduler
        self.queue_waiting.set(sch.num_waiting)
        self.queue_running.set(sch.num_running)
        self.queue_swapped.set(sch.num_swapped)
        self.g_queue.set(sch.num_waiting)
        self.requests_active.set(len(engine.requests))
        self.g_active.set(len(engine.requests))
        bm = engine.bm
        self.kv_usage.set(bm.gpu_usage())
        self.block_usage.set(bm.num_gpu_blocks - bm.num_free_gpu_blocks())
        st = bm.stats()
        q, h = st["prefix_block_queries"], st["prefix_block_hits"]
        dq, dh = q - self._last_prefix[0], h - self._last_prefix[1]
        if dh:
            self.prefix_hits.inc(dh)
        if dq - dh > 0:
            self.prefix_misses.inc(dq - dh)
        self._last_prefix = (q, h)
        if sch.num_preemptions > self._last_preempt:
            self.preemptions.inc(sch.num_preemptions - self._last_preempt)
            self._last_preempt = sch.num_preemptions

    def on_request_finished(self, out, endpoint: str = "completions", status: str = "success") -> None:
        if out is not None and any(c.finish_reason == "abort" and str(c.stop_reason or "").startswith("error:")
                                   for c in out.outputs):
            status = "error"                   # ended by a failure of its own post-processing
            self.errors.labels("request_failed").inc()
        self.requests_total.labels(status).inc()
        self.g_requests.labels(status, self.model, endpoint).inc()
        m = out.metrics if out is not None else None
        if m is None:
            return
        if m.ttft is not None:
            self.ttft.observe(m.ttft)
        if m.tpot is not None:
            self.itl.observe(m.tpot)
            self.g_token_latency.observe(m.tpot)
        if m.e2e_latency is not None:
            self.request_latency.observe(m.e2e_latency)
            self.g_latency.labels(endpoint).observe(m.e2e_latency)
        if m.queue_time is not None:
            self.queue_wait_time.observe(m.queue_time)

    def on_request_params(self, params) -> None:
        self.temperature.observe(params.temperature)
        self.top_p.observe(params.top_p)

    def export(self) -> bytes:
        self.uptime.set(time.time() - self._t0)
        try:
            import torch
            if torch.cuda.is_available():
                for i in range(torch.cuda.device_count()):
                    self.gpu_memory.labels(str(i)).set(torch.cuda.memory_allocated(i))
                    self.g_memory.labels(f"gpu{i}").set(torch.cuda.memory_allocated(i))
        except Exception:  # noqa: BLE001
            pass
        return generate_latest(self.registry)


class Timer:
    """Context manager counterpart of the reference's `time_block!` macro
    (crates/rusteeze-metrics/src/lib.rs:117-129): observes elapsed seconds."""

    def __init__(self, hist: Histogram, *labels):
        self.h = hist.labels(*labels) if labels else hist

    def __enter__(self):
        self.t = time.perf_counter()
        return self

    def __exit__(self, *exc):
        self.h.observe(time.perf_counter() - self.t)
        return False
