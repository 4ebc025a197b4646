"""Latency-SLO batch-size controller.

Counterpart of crates/rusteeze-engine/src/batch_optimizer.rs (unused there):
an exponential moving average of step latency; if it exceeds 1.2x the
target the running-batch cap shrinks by 3/4, if it stays under 0.6x it
grows by 5/4, within [min, max] (batch_optimizer.rs:116-169).  Attached to
the engine as a step observer, it adjusts `scheduler.cfg.max_num_seqs`
live, so operators can trade throughput for inter-token latency.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class BatchOptimizerConfig:
    target_latency_s: float = 0.050
    ema_alpha: float = 0.2
    min_batch: int = 1
    max_batch: int = 256
    high_water: float = 1.2
    low_water: float = 0.6
    shrink: float = 0.75
    grow: float = 1.25
    cooldown_steps: int = 8


class BatchOptimizer:
    def __init__(self, cfg: BatchOptimizerConfig | None = None):
        self.cfg = cfg or BatchOptimizerConfig()
        self.ema: float | None = None
        self.batch = self.cfg.max_batch
        self._since_change = 0
        self.adjustments = 0

    def observe(self, latency_s: float) -> int:
        c = self.cfg
        self.ema = latency_s if self.ema is None else (1 - c.ema_alpha) * self.ema + c.ema_alpha * latency_s
        self._since_change += 1
        if self._since_change >= c.cooldown_steps:
            new = self.batch
            if self.ema > c.high_water * c.target_latency_s:
                new = max(c.min_batch, int(self.batch * c.shrink))
            elif self.ema < c.low_water * c.target_latency_s:
                new = min(c.max_batch, max(self.batch + 1, int(self.batch * c.grow)))
            if new != self.batch:
                self.batch = new
                self.adjustments += 1
                self._since_change = 0
        return self.batch

    def attach(self, engine) -> "BatchOptimizer":
        self.cfg.max_batch = min(self.cfg.max_batch, engine.sched_cfg.max_num_seqs)
        self.batch = self.cfg.max_batch

        def obs(eng, so, step_s):
            eng.scheduler.cfg.max_num_seqs = self.observe(step_s)

        engine.observers.append(obs)
        return self
