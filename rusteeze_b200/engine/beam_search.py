"""Beam search over the paged engine.

The reference declares beam search in its sampling parameters
(crates/rusteeze-core/src/sampling.rs:76-80,206-213: `use_beam_search`, `best_of` as the
width, `length_penalty`, `early_stopping`; validation at sampling.rs:370-380) and a
per-sequence `beam_score` (crates/rusteeze-core/src/sequence.rs:133), but its engine never
runs a search.  Here a request with `use_beam_search` keeps W = `best_of` live beams, one
engine sequence each:

  * a step samples one row per live beam; the sampler returns that beam's 2W most likely
    next tokens after logit bias, min_tokens masking and penalties, as log-probabilities
    (a greedy row with `logprobs` = 2W);
  * a candidate scores the beam's cumulative logprob plus the token's logprob; the best
    2W candidates over all beams are walked in order: one ending in EOS or a stop token id
    becomes a finished hypothesis if it ranks among the first W, any other becomes a live
    beam until W are chosen;
  * a parent chosen k > 1 times is forked k - 1 times (the block manager shares its KV
    blocks copy-on-write), a parent chosen 0 times is freed;
  * hypotheses rank by cumulative logprob / (output tokens, EOS included) ** length_penalty,
    and at most W are kept;
  * early stopping: `true` ends the search once W hypotheses are finished; `false` needs in
    addition that the best live beam, scored at its current length, cannot beat the W-th
    hypothesis; `never` that it cannot beat it at the longest length allowed;
  * the request's outputs are the n best hypotheses, index 0 the best.

Beams advance in lock step.  If a step samples only some live beams (the others were
preempted or did not fit the step's budgets), the sampled beams' step is undone: the KV
slot of their last token is written again by a later step, and the request waits until all
its beams sample in one step.  After `MAX_LAG` such steps in a row the beams that did not
sample are dropped, so a cache too small for W beams narrows the search instead of
stalling it.
"""
from __future__ import annotations

import copy
import math
from typing import Dict, List, Optional, Tuple

from rusteeze_b200.core.sampling_params import EarlyStoppingMode, SamplingParams
from rusteeze_b200.core.types import RequestStatus

MAX_LAG = 64
_MASKED = -1e20


def beam_score(cumulative_logprob: float, num_output_tokens: int, length_penalty: float) -> float:
    """cumulative logprob / L ** length_penalty, with L ** length_penalty taken in log space
    so that no penalty overflows (an infinite divisor gives 0, a vanishing one -inf)."""
    e = length_penalty * math.log(max(1, num_output_tokens))
    if e > 700.0:
        return 0.0
    if e < -700.0:
        return -math.inf if cumulative_logprob < 0 else 0.0
    return cumulative_logprob / math.exp(e)


class BeamState:
    """Search state of one request: width, the sampling parameters of its rows, and the
    finished hypotheses as (score, sequence), best first."""

    __slots__ = ("width", "row_params", "finished", "done", "lag", "max_output")

    def __init__(self, params: SamplingParams, max_output: int):
        self.width = int(params.best_of)
        # the rows are greedy rows whose logprob table is the 2W best tokens; built without
        # re-validation (the table is larger than a user may ask for)
        rp = copy.copy(params)
        rp.use_beam_search = False
        rp.temperature = 0.0
        rp.n = rp.best_of = 1
        rp.logprobs = 2 * self.width
        self.row_params = rp
        self.finished: List[Tuple[float, object]] = []
        self.done = False
        self.lag = 0
        self.max_output = max_output

    def add_hypothesis(self, seq, length_penalty: float) -> Optional[object]:
        """Adds a finished sequence; returns the one that fell out of the best W (or None)."""
        sc = beam_score(seq.cumulative_logprob, seq.num_generated, length_penalty)
        self.finished.append((sc, seq))
        self.finished.sort(key=lambda t: (-t[0], t[1].seq_id))
        if len(self.finished) > self.width:
            return self.finished.pop()[1]
        return None

    def worst_kept(self) -> float:
        return self.finished[-1][0] if len(self.finished) >= self.width else float("-inf")

    def is_done(self, best_live_cum: float, live_len: int, params: SamplingParams) -> bool:
        if len(self.finished) < self.width:
            return False
        mode = EarlyStoppingMode(params.early_stopping)
        if mode == EarlyStoppingMode.TRUE:
            return True
        lp = params.length_penalty
        if mode == EarlyStoppingMode.NEVER and lp > 0:
            best = beam_score(best_live_cum, self.max_output, lp)
        else:
            best = beam_score(best_live_cum, live_len, lp)
        return self.worst_kept() >= best


class BeamSearcher:
    """The engine side of beam search: the step that turns a request's sampled rows into
    its next set of beams."""

    def __init__(self, engine):
        self.eng = engine

    def start(self, req) -> None:
        p = req.params
        cap = self.eng.max_model_len - len(req.prompt_token_ids)
        max_out = min(p.max_tokens, cap) if p.max_tokens is not None else cap
        req.beam = BeamState(p, max(1, max_out))

    def _is_stop_token(self, req, tok: int) -> bool:
        p = req.params
        return (not p.ignore_eos and tok in self.eng.eos_ids) or tok in p.stop_token_ids

    def _prune(self, s) -> None:
        """A beam that leaves the search: KV freed, never reported."""
        eng = self.eng
        if not s.is_finished():
            eng.scheduler.remove(s)
            eng.bm.free(s.seq_id)
        s.status = RequestStatus.FINISHED_ABORTED
        s.finish_reason = None
        s.pruned = True

    @staticmethod
    def _keep(req, s) -> None:
        """A finished beam (stop, length) or hypothesis joins the ranked list."""
        out = req.beam.add_hypothesis(s, req.params.length_penalty)
        if out is not None:
            out.pruned = True

    def step(self, req, entries: List[Tuple[object, object, Optional[Dict[int, float]]]], now: float) -> None:
        """entries: (sequence, its scheduled share, top-logprob table) for every beam of
        `req` sampled this step."""
        eng, st, p = self.eng, req.beam, req.params
        if st.done:
            return
        live = [s for s in req.seqs if not s.is_finished()]
        sampled = {s.seq_id for s, _, _ in entries}
        missing = [s for s in live if s.seq_id not in sampled]
        if missing:
            if st.lag < MAX_LAG:
                st.lag += 1
                for s, ss, _ in entries:          # undo: this token's KV is written again later
                    s.num_computed = ss.ctx + ss.num_new - 1
                return
            for s in missing:
                self._prune(s)
        st.lag = 0
        W = st.width
        cands = []
        for s, _, top in entries:
            for tok, lp in (top or {}).items():
                if lp > _MASKED:
                    cands.append((s.cumulative_logprob + lp, s, int(tok), float(lp)))
        cands.sort(key=lambda c: (-c[0], c[1].index, c[2]))
        chosen: List[Tuple[object, int, float]] = []
        for rank, (_, s, tok, lp) in enumerate(cands[:2 * W]):
            if self._is_stop_token(req, tok) and s.num_generated + 1 >= p.min_tokens:
                if rank < W:
                    h = s.fork_copy(index=-1, with_kv=False)
                    h.append_token(tok, lp, self._table(p, s, tok, lp, entries))
                    if not req.defer_text and h.detok is not None:
                        h.output_text += h.detok.step(tok)
                        h.detok_n += 1
                    h.status = RequestStatus.FINISHED_STOPPED
                    h.finish_reason = "stop"
                    h.stop_reason = tok if tok in p.stop_token_ids else None
                    req.seqs.append(h)
                    eng._register_seq(req, h)
                    self._keep(req, h)
                continue
            chosen.append((s, tok, lp))
            if len(chosen) == W:
                break
        uses: Dict[int, int] = {}
        for s, _, _ in chosen:
            uses[s.seq_id] = uses.get(s.seq_id, 0) + 1
        for s, _, _ in entries:
            if s.seq_id not in uses:
                self._prune(s)
        # forks first (a child copies the parent's tokens before the parent grows)
        targets = []
        first = set()
        for s, tok, lp in chosen:
            if s.seq_id in first:
                c = s.fork_copy(index=len(req.seqs), with_kv=True)
                eng.bm.fork(s.seq_id, c.seq_id)
                req.seqs.append(c)
                eng._register_seq(req, c)
                eng.scheduler.add_running(c)
                targets.append((c, tok, lp, s))
            else:
                first.add(s.seq_id)
                targets.append((s, tok, lp, s))
        for t, tok, lp, parent in targets:
            t.append_token(tok, lp, self._table(p, parent, tok, lp, entries))
            eng.stats_counters["generation_tokens"] += 1
            eng._check_stop(t, tok)
            if t.is_finished():
                self._keep(req, t)
        req.metrics.last_token_time = now
        if req.metrics.first_token_time is None:
            req.metrics.first_token_time = now
        req.metrics.num_generated = max((s.num_generated for s in req.seqs), default=0)
        live = [s for s in req.seqs if not s.is_finished()]
        if not live:
            st.done = True
            return
        best = max(live, key=lambda s: s.cumulative_logprob)
        if st.is_done(best.cumulative_logprob, best.num_generated, p):
            for s in live:
                self._prune(s)
            st.done = True

    @staticmethod
    def _table(p: SamplingParams, s, tok: int, lp: float, entries) -> Optional[Dict[int, float]]:
        """The logprob entry of an output token: the user's top `logprobs` of the parent's
        row plus the chosen token."""
        if p.logprobs is None:
            return None
        top = next((t for q, _, t in entries if q is s), None) or {}
        d = dict(sorted(top.items(), key=lambda kv: -kv[1])[:p.logprobs])
        d[tok] = lp
        return d
