"""Continuous-batching iteration scheduler.

What the reference's scheduler does (crates/rusteeze-engine/src/
scheduler.rs:142-215): retire finished sequences, give every running
sequence one decode token (highest priority first) within the token and
sequence budgets, preempt what does not fit, then admit waiting prompts FCFS
within the token budget.  Its gaps -- no KV-block availability check, no
chunked prefill, preempted sequences never come back -- are closed here:

  * every admission and every decode checks free KV blocks in the C++
    block manager (including the copy-on-write block of forked sequences);
  * prompts are split into chunks that fit the per-step token budget
    (`enable_chunked_prefill`), and a chunked prompt keeps its place;
  * preemption is either RECOMPUTE (free the blocks, re-prefill later; the
    reference's default, scheduler.rs:48-83) or SWAP (KV moved to CPU
    blocks and swapped back in before new prompts are admitted);
  * waiting order is FCFS, shortest-job-first or priority
    (crates/rusteeze-config/src/engine.rs scheduling policy knob);
  * a watermark of free blocks is kept so that running sequences can grow.

The output orders decodes (one new token each) before prefill chunks, which
is the layout the attention kernels expect.
"""
from __future__ import annotations

import enum
from collections import deque
from dataclasses import dataclass, field
from typing import Deque, List, Tuple

from rusteeze_b200.core.types import RequestStatus
from rusteeze_b200.engine.sequence import Sequence


class PreemptionMode(str, enum.Enum):
    RECOMPUTE = "recompute"
    SWAP = "swap"


class SchedulingPolicy(str, enum.Enum):
    FCFS = "fcfs"
    SJF = "sjf"
    PRIORITY = "priority"


@dataclass
class SchedulerConfig:
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    max_model_len: int = 8192
    enable_chunked_prefill: bool = True
    preemption_mode: PreemptionMode = PreemptionMode.RECOMPUTE
    policy: SchedulingPolicy = SchedulingPolicy.FCFS
    watermark: float = 0.01
    num_lookahead_slots: int = 0        # speculative decoding: k draft tokens
    max_prefill_seqs: int = 64          # bound on prefill chunks per step


class ScheduledSeq:
    """One sequence's share of a step (a plain slotted class: thousands are built per step)."""
    __slots__ = ("seq", "ctx", "num_new", "sample", "num_samples", "pend_row")

    def __init__(self, seq: Sequence, ctx: int, num_new: int, sample: bool, num_samples: int = 1,
                 pend_row: int = -1):
        self.seq = seq
        self.ctx = ctx                  # tokens with KV before this step
        self.num_new = num_new          # tokens computed this step
        self.sample = sample            # logits of the last new token are sampled
        self.num_samples = num_samples
        self.pend_row = pend_row        # async scheduling: row of the previous step's samples that is this step's input

    def __repr__(self) -> str:
        return (f"ScheduledSeq(seq={self.seq.seq_id}, ctx={self.ctx}, num_new={self.num_new}, "
                f"sample={self.sample}, num_samples={self.num_samples}, pend_row={self.pend_row})")


@dataclass
class SchedulerOutput:
    decodes: List[ScheduledSeq] = field(default_factory=list)
    prefills: List[ScheduledSeq] = field(default_factory=list)
    blocks_to_copy: List[Tuple[int, int]] = field(default_factory=list)
    blocks_to_swap_in: List[Tuple[int, int]] = field(default_factory=list)
    blocks_to_swap_out: List[Tuple[int, int]] = field(default_factory=list)
    preempted: List[Sequence] = field(default_factory=list)
    num_batched_tokens: int = 0

    @property
    def scheduled(self) -> List[ScheduledSeq]:
        return self.decodes + self.prefills

    def is_empty(self) -> bool:
        return not self.decodes and not self.prefills


def _sched_key(s: Sequence):
    """Running order: highest priority, then oldest request, then sequence id (fixed for a
    sequence's life, so it is computed once)."""
    k = s.sched_key
    if k is None:
        r = s.request
        k = s.sched_key = (-r.priority, r.arrival_time, s.seq_id)
    return k


class Scheduler:
    def __init__(self, cfg: SchedulerConfig, block_manager):
        self.cfg = cfg
        self.bm = block_manager
        self.waiting: Deque[Sequence] = deque()
        self.running: List[Sequence] = []
        self.swapped: Deque[Sequence] = deque()
        self.num_preemptions = 0
        self.ignored: List[Sequence] = []      # too long to ever run; the engine reports and drops them
        self._watermark_blocks = max(1, int(cfg.watermark * self.bm.num_gpu_blocks))
        self._bs = self.bm.block_size

    # ------------------------------------------------------------------ queue ops
    def add(self, seq: Sequence) -> None:
        seq.status = RequestStatus.WAITING
        self.waiting.append(seq)

    def add_running(self, seq: Sequence) -> None:
        """A forked child joins the running set directly."""
        seq.status = RequestStatus.RUNNING
        self.running.append(seq)

    def remove(self, seq: Sequence) -> None:
        for q in (self.running,):
            if seq in q:
                q.remove(seq)
        for dq in (self.waiting, self.swapped):
            try:
                dq.remove(seq)
            except ValueError:
                pass

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running or self.swapped)

    @property
    def num_waiting(self) -> int:
        return len(self.waiting)

    @property
    def num_running(self) -> int:
        return len(self.running)

    @property
    def num_swapped(self) -> int:
        return len(self.swapped)

    # ------------------------------------------------------------------ helpers
    def _key(self, s: Sequence):
        return _sched_key(s)

    def _sort_waiting(self) -> None:
        pol = self.cfg.policy
        if pol == SchedulingPolicy.FCFS:
            return  # deque order is arrival order; preempted seqs are re-queued at the front
        if pol == SchedulingPolicy.SJF:
            key = lambda s: (s.total_len, s.request.arrival_time)  # noqa: E731
        else:
            key = lambda s: (-s.request.priority, s.request.arrival_time)  # noqa: E731
        self.waiting = deque(sorted(self.waiting, key=key))

    def _preempt(self, seq: Sequence, out: SchedulerOutput) -> None:
        self.num_preemptions += 1
        out.preempted.append(seq)
        if self.cfg.preemption_mode == PreemptionMode.SWAP and self.bm.can_swap_out(seq.seq_id):
            out.blocks_to_swap_out.extend(self.bm.swap_out(seq.seq_id))
            seq.status = RequestStatus.SWAPPED
            self.swapped.append(seq)
        else:
            self.bm.free(seq.seq_id)
            seq.reset_for_recompute()
            self.waiting.appendleft(seq)

    def _drop_too_long(self, seq: Sequence) -> None:
        """A running sequence whose next step would need more KV blocks than the GPU
        cache has: free it and report it finished by length."""
        self.bm.free(seq.seq_id)
        seq.status = RequestStatus.FINISHED_IGNORED
        seq.finish_reason = "length"
        self.ignored.append(seq)

    def _finishes_with_pending(self, seq: Sequence) -> bool:
        p = seq.request.params
        n = seq.num_generated + seq.pending
        return (p.max_tokens is not None and n >= p.max_tokens) or seq.total_len >= self.cfg.max_model_len

    def _lookahead(self, seq: Sequence) -> int:
        return self.cfg.num_lookahead_slots if not seq.is_prefill else 0

    # ------------------------------------------------------------------ main
    def schedule(self) -> SchedulerOutput:
        cfg, bm = self.cfg, self.bm
        out = SchedulerOutput()
        token_budget = cfg.max_num_batched_tokens
        seq_budget = cfg.max_num_seqs

        # 1. running sequences, highest priority / oldest first.  running[i:end] is the
        # queue still to visit; preemption takes the lowest priority one from its end.
        running = self.running
        running.sort(key=_sched_key)
        kept: List[Sequence] = []
        bs, ngpu = self._bs, bm.num_gpu_blocks
        la_decode = cfg.num_lookahead_slots
        decodes, prefills = out.decodes, out.prefills
        i, end = 0, len(running)
        while i < end:
            seq = running[i]
            i += 1
            if seq.pending and self._finishes_with_pending(seq):
                kept.append(seq)            # its in-flight token is its last: nothing to schedule
                continue
            total = len(seq.token_ids) + seq.pending
            nc = seq.num_computed
            prefill = total - nc > 1
            if prefill:
                n = min(total - nc, token_budget)
                if n <= 0 or seq_budget <= 0:
                    kept.append(seq)        # keeps its blocks, continues next step
                    continue
                la = 0
            else:
                n = 1
                la = la_decode
                if token_budget < 1 + la or seq_budget <= 0:
                    self._preempt(seq, out)
                    continue
            target = nc + n + la
            if (target + bs - 1) // bs > ngpu:
                # its KV can never fit the whole cache: the sequence ends here ("length")
                self._drop_too_long(seq)
                continue
            cow = bm.try_grow(seq.seq_id, target, nc)
            while cow is None and i < end:
                end -= 1
                self._preempt(running[end], out)  # lowest priority goes first
                cow = bm.try_grow(seq.seq_id, target, nc)
            if cow is None:
                self._preempt(seq, out)
                continue
            if cow:
                out.blocks_to_copy.extend(cow)
            done_prompt = nc + n >= total
            ss = ScheduledSeq(seq, nc, n, done_prompt, self._num_samples(seq) if done_prompt else 1)
            (prefills if n > 1 or prefill else decodes).append(ss)
            token_budget -= n + (la if n == 1 else 0)
            seq_budget -= 1
            kept.append(seq)
        self.running = kept

        # 2. swapped sequences come back before new prompts (unless we just preempted)
        if not out.preempted:
            while self.swapped and seq_budget > 0 and token_budget > 0:
                seq = self.swapped[0]
                held = len(bm.block_table(seq.seq_id))
                # the watermark reserve only applies while there is room for it
                need = held + (self._watermark_blocks if held + self._watermark_blocks <= bm.num_gpu_blocks else 0)
                if need > bm.num_free_gpu_blocks():
                    break
                self.swapped.popleft()
                out.blocks_to_swap_in.extend(bm.swap_in(seq.seq_id))
                seq.status = RequestStatus.RUNNING
                n = min(seq.remaining, token_budget) if seq.is_prefill else 1
                target = seq.num_computed + n + self._lookahead(seq)
                if bm.blocks_to_grow(seq.seq_id, target, seq.num_computed) > bm.num_free_gpu_blocks():
                    self.running.append(seq)
                    continue
                out.blocks_to_copy.extend(bm.ensure_capacity(seq.seq_id, target, seq.num_computed))
                done_prompt = seq.num_computed + n >= seq.total_len
                # a prompt swapped out mid-prefill forks its best_of samples here like anywhere else
                ss = ScheduledSeq(seq, seq.num_computed, n, sample=done_prompt,
                                  num_samples=self._num_samples(seq) if done_prompt else 1)
                (out.prefills if n > 1 or seq.is_prefill else out.decodes).append(ss)
                token_budget -= n
                seq_budget -= 1
                self.running.append(seq)

        # 3. waiting prompts (or recompute-preempted sequences)
        if not self.swapped:
            self._sort_waiting()
            n_prefill = len(out.prefills)
            while self.waiting and seq_budget > 0 and token_budget > 0 and n_prefill < cfg.max_prefill_seqs:
                seq = self.waiting[0]
                if seq.pending:
                    break                   # preempted this step with a token still in flight
                if (seq.total_len > cfg.max_model_len or
                        bm.blocks_for(seq.total_len + 1) > bm.num_gpu_blocks):
                    # longer than the model, or its KV (with the first sampled token) could
                    # never fit the whole GPU cache: report it instead of waiting forever
                    self.waiting.popleft()
                    seq.status = RequestStatus.FINISHED_IGNORED
                    seq.finish_reason = "length"
                    self.ignored.append(seq)
                    continue
                toks = seq.tokens_np()
                cached = bm.cached_prefix_len(toks) if not bm.has_seq(seq.seq_id) else seq.num_computed
                remaining = seq.total_len - cached
                if (not cfg.enable_chunked_prefill and remaining > token_budget
                        and remaining <= cfg.max_num_batched_tokens):
                    break                   # waits for a step with room for all of it
                # (longer than any step's budget: without chunks it could never run, so it
                # is chunked even with chunked prefill off -- a long prompt, or a sequence
                # that grew past the budget and was preempted by recompute)
                n = min(remaining, token_budget)
                need = bm.blocks_needed_for_prompt(toks, cached + n)
                if need + self._watermark_blocks > bm.num_free_gpu_blocks():
                    break
                self.waiting.popleft()
                if not bm.has_seq(seq.seq_id):
                    got = bm.allocate_prompt(seq.seq_id, toks)
                    seq.num_computed = got
                    seq.num_cached = got
                    if seq.request.metrics.first_scheduled_time is None:
                        import time
                        seq.request.metrics.first_scheduled_time = time.monotonic()
                out.blocks_to_copy.extend(bm.ensure_capacity(seq.seq_id, seq.num_computed + n,
                                                             seq.num_computed))
                seq.status = RequestStatus.RUNNING
                done_prompt = seq.num_computed + n >= seq.total_len
                out.prefills.append(ScheduledSeq(seq, seq.num_computed, n, sample=done_prompt,
                                                 num_samples=self._num_samples(seq) if done_prompt else 1))
                self.running.append(seq)
                token_budget -= n
                seq_budget -= 1
                n_prefill += 1

        # decodes that are really single-token prompt tails stay as "prefill"
        # only if they have more than one token; re-split for the kernel layout
        out.num_batched_tokens = sum(s.num_new for s in out.decodes) + sum(s.num_new for s in out.prefills)
        return out

    def _num_samples(self, seq: Sequence) -> int:
        r = seq.request
        # beam search samples one row per beam; its search forks the beams
        if r.forked or r.num_target_seqs == 1 or seq.num_generated > 0 or r.beam is not None:
            return 1
        return r.num_target_seqs
