"""Sequences and requests (sequence groups).

Counterpart of crates/rusteeze-engine/src/sequence.rs:70-429 (Sequence,
SequenceGroup, stop handling) and crates/rusteeze-core/src/sequence.rs:80-517
(timing: TTFT, ITL).  A request with n > 1 (or best_of > n) owns several
sequences that share the prompt's KV blocks copy-on-write after the prompt is
prefilled.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from rusteeze_b200.core.outputs import CompletionOutput, RequestOutput
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.core.types import RequestMetrics, RequestStatus

_seq_ids = itertools.count(1)


def _stop_prefix_len(text: str, stops) -> int:
    """Length of the longest suffix of `text` that is a proper prefix of a stop string."""
    best = 0
    for st in stops:
        for k in range(min(len(st) - 1, len(text)), best, -1):
            if text.endswith(st[:k]):
                best = k
                break
    return best


class Sequence:
    __slots__ = ("seq_id", "request", "prompt_len", "token_ids", "status", "num_computed",
                 "num_cached", "logprobs", "cumulative_logprob", "output_text", "stop_reason",
                 "detok", "_buf", "index", "finish_reason", "rng_offset",
                 "mirostat_mu", "spec_draft", "pending", "detok_n", "sched_key", "pruned", "guide")

    def __init__(self, request: "Request", prompt_token_ids: List[int], index: int = 0):
        self.seq_id = next(_seq_ids)
        self.request = request
        self.index = index
        self.prompt_len = len(prompt_token_ids)
        self.token_ids: List[int] = list(prompt_token_ids)
        self.status = RequestStatus.WAITING
        self.num_computed = 0          # tokens whose KV is in the cache
        self.num_cached = 0            # of those, reused from the prefix cache
        self.logprobs: List[Dict[int, float]] = []
        self.cumulative_logprob = 0.0
        self.output_text = ""
        self.stop_reason = None
        self.finish_reason: Optional[str] = None
        self.detok = None
        self.detok_n = 0               # output tokens already fed to the detokenizer
        self.sched_key = None          # running-queue order, set by the scheduler
        # int64 mirror of token_ids with room to grow: batch building slices it
        # without converting the Python list every step
        self._buf = np.empty(max(16, self.prompt_len + min(request.params.max_tokens or 256, 4096) + 8
                                 if request is not None else self.prompt_len + 16), dtype=np.int64)
        self._buf[:self.prompt_len] = prompt_token_ids
        self.rng_offset = 0
        self.mirostat_mu = None
        self.spec_draft: List[int] = []
        # tokens sampled by steps still running on the GPU (asynchronous
        # scheduling): their KV position is already reserved, their value is
        # only on the device until the step's results are applied
        self.pending = 0
        self.pruned = False            # a beam that left the search: never reported
        self.guide = None              # guided decoding: position in the constraint's automaton

    def fork_copy(self, index: int, with_kv: bool) -> "Sequence":
        """A new sequence with this one's tokens, logprobs, text and detokenizer state
        (beam search); `with_kv` also copies the KV counters, for a child that shares the
        parent's blocks through the block manager's fork."""
        c = Sequence(self.request, self.token_ids[:self.prompt_len], index)
        n = len(self.token_ids)
        if c._buf.shape[0] < self._buf.shape[0]:
            c._buf = np.empty_like(self._buf)
        c._buf[:n] = self._buf[:n]
        c.token_ids = list(self.token_ids)
        c.logprobs = list(self.logprobs)
        c.cumulative_logprob = self.cumulative_logprob
        c.output_text = self.output_text
        c.detok = self.detok.clone() if self.detok is not None else None
        c.detok_n = self.detok_n
        c.mirostat_mu = self.mirostat_mu
        c.guide = self.guide.copy() if self.guide is not None else None
        if with_kv:
            c.num_computed, c.num_cached = self.num_computed, self.num_cached
        return c

    # ------------------------------------------------------------------
    @property
    def output_token_ids(self) -> List[int]:
        return self.token_ids[self.prompt_len:]

    @property
    def num_generated(self) -> int:
        return len(self.token_ids) - self.prompt_len

    @property
    def total_len(self) -> int:
        """Tokens of the sequence including in-flight (pending) samples."""
        return len(self.token_ids) + self.pending

    @property
    def is_prefill(self) -> bool:
        """More than one token still lacks KV (prompt or recompute after preemption)."""
        return self.total_len - self.num_computed > 1

    @property
    def remaining(self) -> int:
        return self.total_len - self.num_computed

    def tokens_np(self) -> np.ndarray:
        """View of all tokens (prompt + generated) as int64; valid until the next append."""
        return self._buf[:len(self.token_ids)]

    def append_token(self, tok: int, logprob: Optional[float] = None,
                     top: Optional[Dict[int, float]] = None) -> None:
        tok = int(tok)
        n = len(self.token_ids)
        if n >= self._buf.shape[0]:
            nb = np.empty(2 * self._buf.shape[0], dtype=np.int64)
            nb[:n] = self._buf[:n]
            self._buf = nb
        self._buf[n] = tok
        self.token_ids.append(tok)
        if logprob is not None:
            self.cumulative_logprob += float(logprob)
        if top is not None:
            self.logprobs.append(top)

    def is_finished(self) -> bool:
        return self.status.is_finished

    def materialize_text(self) -> None:
        """Detokenises the output tokens not yet fed to the detokenizer (outputs whose
        text is deferred until it is read)."""
        n = len(self.token_ids) - self.prompt_len
        if self.detok is not None and self.detok_n < n:
            self.output_text += self.detok.extend(self.token_ids[self.prompt_len + self.detok_n:])
            self.detok_n = n

    def reset_for_recompute(self) -> None:
        """Preemption by recompute: drop all KV; prompt+generated get re-prefilled."""
        self.num_computed = 0
        self.num_cached = 0
        self.status = RequestStatus.WAITING


@dataclass
class Request:
    request_id: str
    prompt: Optional[str]
    prompt_token_ids: List[int]
    params: SamplingParams
    arrival_time: float
    priority: int = 0
    seqs: List[Sequence] = field(default_factory=list)
    metrics: RequestMetrics = None
    forked: bool = False
    lora: Optional[str] = None
    beam: Optional[object] = None          # beam search state (engine/beam_search.py)
    prompt_lp: Optional[list] = None       # prompt logprobs, once scored
    # streaming state
    sent_text_len: Dict[int, int] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.metrics is None:
            self.metrics = RequestMetrics(arrival_time=self.arrival_time)
        if not self.seqs:
            self.seqs = [Sequence(self, self.prompt_token_ids, 0)]
        # per-step outputs for streaming consumers; final-only requests without stop
        # strings detokenise once, when their output is built
        self.stream = self.params.output_kind == "delta"
        self.defer_text = not self.stream and not self.params.stop

    @property
    def num_target_seqs(self) -> int:
        return self.params.best_of

    def is_finished(self) -> bool:
        if self.beam is not None:
            return all(s.is_finished() for s in self.seqs)
        # with best_of > 1 the children are forked when the prompt's last
        # chunk is sampled; until then the request cannot be finished
        return (self.forked or self.num_target_seqs == 1) and all(s.is_finished() for s in self.seqs)

    def live_seqs(self) -> List[Sequence]:
        return [s for s in self.seqs if not s.is_finished()]

    def _beam_outputs(self) -> List[Sequence]:
        """The n best finished hypotheses (or, while the search runs, the n best live beams),
        best first."""
        n = self.params.n
        if self.is_finished():
            seqs = [s for _, s in self.beam.finished][:n]
            return seqs or [s for s in self.seqs if not s.pruned][:n]
        return sorted(self.live_seqs(), key=lambda s: -s.cumulative_logprob)[:n]

    def to_output(self, delta: bool = False) -> RequestOutput:
        p = self.params
        seqs = self.seqs
        if self.beam is not None:
            seqs = self._beam_outputs()
        elif self.is_finished() and len(seqs) > p.n:
            # best_of > n: keep the n sequences with the highest cumulative logprob
            seqs = sorted(seqs, key=lambda s: s.cumulative_logprob, reverse=True)[: p.n]
        outs = []
        deltas = []
        beam_fin = self.beam is not None and self.is_finished()
        for rank, s in enumerate(seqs):
            if self.defer_text:
                s.materialize_text()
            text = s.output_text
            idx = rank if self.beam is not None else s.index
            outs.append(CompletionOutput(index=idx, text=text, token_ids=s.output_token_ids,
                                         cumulative_logprob=s.cumulative_logprob if p.logprobs is not None else None,
                                         logprobs=s.logprobs if p.logprobs is not None else None,
                                         finish_reason=s.finish_reason, stop_reason=s.stop_reason))
            prev = self.sent_text_len.get(idx, 0)
            if self.beam is not None and not beam_fin:
                deltas.append("")          # beams are re-ranked every step: text goes out at the end
                continue
            # a running sequence's text may end in the start of a stop string, which the next
            # token could complete (and the stop string is then cut from the output): hold
            # that suffix back so a stream never sends text it would have to retract
            end = len(text) if s.is_finished() or not p.stop else len(text) - _stop_prefix_len(text, p.stop)
            end = max(end, prev)
            deltas.append(text[prev:end])
            if delta:
                self.sent_text_len[idx] = end
        return RequestOutput(request_id=self.request_id, prompt=self.prompt,
                             prompt_token_ids=self.prompt_token_ids, outputs=outs,
                             finished=self.is_finished(), metrics=self.metrics,
                             num_cached_tokens=max((s.num_cached for s in self.seqs), default=0),
                             delta_text=deltas, prompt_logprobs=self.prompt_lp)
