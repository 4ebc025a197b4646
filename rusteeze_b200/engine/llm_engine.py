"""The engine: request intake, the step loop, stop handling, outputs.

Counterpart of crates/rusteeze-engine/src/engine.rs.  The reference's
`Engine::step` (engine.rs:357-435) schedules, builds a batch, and hands the
worker a closure that writes ZERO logits (engine.rs:418-427), so it always
samples token 0; `generate` runs a single step per request (engine.rs:292).
Here `step()` runs the real model: schedule -> (swap/CoW block copies) ->
batch build -> forward (CUDA graph for pure decode) -> on-device sampling ->
append tokens -> stop checks (EOS unless ignore_eos, stop token ids, stop
strings through the incremental detokenizer, max_tokens, max_model_len) ->
free blocks of finished sequences -> RequestOutputs.  `LLM.generate` drives
steps until every request finishes.

Finish reasons: "stop" (EOS/stop token/stop string), "length" (max_tokens or
context limit), "abort" -- the reference always reports Stop (engine.rs:
497-555).
"""
from __future__ import annotations

import logging
import os
import time
from typing import Callable, Dict, List, Optional, Union

import numpy as np
import torch

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.errors import ContextLengthExceededError, InvalidRequestError
from rusteeze_b200.core.outputs import RequestOutput
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.core.types import RequestStatus, new_request_id
from rusteeze_b200.engine.beam_search import BeamSearcher
from rusteeze_b200.engine.block_manager import make_block_manager
from rusteeze_b200.engine.model_runner import ModelRunner
from rusteeze_b200.engine.sampler import SampleRow, Sampler
from rusteeze_b200.engine.scheduler import (PreemptionMode, Scheduler, SchedulerConfig,
                                            SchedulingPolicy)
from rusteeze_b200.engine.sequence import Request, Sequence
from rusteeze_b200.models.config import ModelConfig, get_preset
from rusteeze_b200.models.loader import build_model
from rusteeze_b200.tokenizer.tokenizer import IncrementalDetokenizer, load_tokenizer
from rusteeze_b200.ops import BLOCK_SIZE
from rusteeze_b200.metrics.logging_setup import nvtx_range

log = logging.getLogger("rusteeze.engine")


class _InFlight:
    """A launched step whose sampled tokens are still on the GPU."""
    __slots__ = ("so", "handle", "owners", "rows_of", "t_launch")

    def __init__(self, so, handle, owners, rows_of, t_launch):
        self.so, self.handle, self.owners, self.rows_of, self.t_launch = so, handle, owners, rows_of, t_launch


def _dtype(name: str, device: str) -> torch.dtype:
    if name in ("auto", "bfloat16", "bf16"):
        return torch.bfloat16 if device.startswith("cuda") else torch.float32
    return {"float32": torch.float32, "fp32": torch.float32, "float16": torch.float16,
            "fp16": torch.float16}[name]


def kv_cache_dtype(name: str, model_dtype: torch.dtype) -> torch.dtype:
    """Element type of the paged KV cache: the model dtype ("auto" or its own name), or fp8
    ("fp8" / "fp8_e4m3": float8_e4m3fn, "fp8_e5m2": float8_e5m2)."""
    n = (name or "auto").lower()
    if n in ("fp8", "fp8_e4m3"):
        return torch.float8_e4m3fn
    if n == "fp8_e5m2":
        return torch.float8_e5m2
    return model_dtype


def swap_blocks(ec, model_config, dtype: torch.dtype, device: str) -> int:
    """Host swap-space blocks for swap preemption.  Every tensor-parallel rank computes
    the same count from the same config (the engine's block manager on rank 0 and each
    rank's host KV cache must agree)."""
    cuda = str(device).startswith("cuda")
    bytes_per_block = model_config.kv_bytes_per_token(torch.finfo(dtype).bits // 8) * BLOCK_SIZE
    n = int(ec.swap_space_gb * (1 << 30) // bytes_per_block)
    if not cuda:
        n = min(n, 1024)
    if ec.scheduling.preemption_mode != "swap" and cuda:
        n = 0
    return n


def resolve_device(name: str) -> str:
    if name == "auto":
        return "cuda:0" if torch.cuda.is_available() else "cpu"
    if name == "cuda":
        return "cuda:0"
    return name


class LLMEngine:
    def __init__(self, config: Config, model=None, model_config: Optional[ModelConfig] = None,
                 tokenizer=None, tp=None, executor=None):
        self.config = config
        mc = config.model
        ec = config.engine
        self.device = resolve_device(mc.device)
        if model is not None:
            self.model_config = model.cfg
        elif model_config is not None:
            self.model_config = model_config
        elif mc.path:
            self.model_config = ModelConfig.from_json_file(mc.path)
        else:
            self.model_config = get_preset(mc.preset or "tiny-llama")
        self.max_model_len = min(mc.max_model_len or self.model_config.max_position_embeddings,
                                 self.model_config.max_position_embeddings)
        self.dtype = _dtype(mc.dtype, self.device)
        if self.device.startswith("cuda"):
            torch.cuda.set_device(torch.device(self.device))
        if model is None:
            model = build_model(self.model_config, dtype=self.dtype, device=self.device, tp=tp,
                                model_dir=mc.path, seed=mc.seed)
            if mc.quantization is not None and mc.quantization.method != "none":
                from rusteeze_b200.models.quant import quantize_model_fp8
                quantize_model_fp8(model, getattr(mc.quantization, "scale_format", "ue8m0"))
        if self.device.startswith("cuda"):
            model.prepare_for_gpu()
        self.model = model
        self.tokenizer = tokenizer or load_tokenizer(mc.tokenizer or mc.path, self.model_config.vocab_size)
        self.model_name = mc.served_name()
        self.eos_ids = tuple(self.model_config.eos_token_id or ([self.tokenizer.eos_token_id]
                                                               if self.tokenizer.eos_token_id is not None else []))
        # KV cache sizing
        self.kv_dtype = kv_cache_dtype(ec.kv_cache_dtype, self.dtype)
        num_gpu_blocks = ec.num_gpu_blocks or self._profile_num_blocks()
        num_cpu_blocks = swap_blocks(ec, self.model_config, self.kv_dtype, self.device)
        self.bm = make_block_manager(BLOCK_SIZE, num_gpu_blocks, num_cpu_blocks, ec.enable_prefix_caching)
        spec = ec.speculative
        self.sched_cfg = SchedulerConfig(
            max_num_seqs=ec.max_num_seqs, max_num_batched_tokens=ec.max_num_batched_tokens,
            max_model_len=self.max_model_len, enable_chunked_prefill=ec.enable_chunked_prefill,
            preemption_mode=PreemptionMode(ec.scheduling.preemption_mode),
            policy=SchedulingPolicy(ec.scheduling.policy),
            num_lookahead_slots=spec.num_speculative_tokens if spec else 0)
        self.scheduler = Scheduler(self.sched_cfg, self.bm)
        self.runner = executor or ModelRunner(
            model, num_gpu_blocks=num_gpu_blocks, num_cpu_blocks=num_cpu_blocks,
            max_num_seqs=ec.max_num_seqs, max_num_batched_tokens=ec.max_num_batched_tokens,
            max_model_len=self.max_model_len, kv_dtype=self.kv_dtype, use_cuda_graph=not ec.enforce_eager,
            seed=mc.seed)
        if self.device.startswith("cuda") and not ec.enforce_eager and hasattr(self.runner, "capture_graphs"):
            from rusteeze_b200.engine.model_runner import decode_graph_buckets
            mx = min(ec.cuda_graph_max_batch or ec.max_num_seqs, ec.max_num_seqs)
            self.runner.capture_graphs(decode_graph_buckets(mx))
        self.requests: Dict[str, Request] = {}
        self.seq_to_request: Dict[int, Request] = {}
        self._rng = np.random.default_rng(mc.seed)
        self.stats_counters = {"steps": 0, "prompt_tokens": 0, "generation_tokens": 0,
                               "requests_finished": 0, "requests_aborted": 0, "requests_failed": 0}
        self.observers: List[Callable] = []
        self._prefix_caching = bool(ec.enable_prefix_caching)
        # device sampling slots (one per live sequence) of the rank that samples
        self._sampler = getattr(self.runner, "sampler", None)
        if self._sampler is not None and self.device.startswith("cuda"):
            self._sampler.max_slots = ec.max_num_seqs + 64
        self.phase_s: Dict[str, float] = {"schedule": 0.0, "postprocess": 0.0}
        # asynchronous scheduling: CUDA engine without speculation over a runner (or a
        # tensor-parallel executor) that can pipeline steps
        self._async = (ec.async_scheduling and self.device.startswith("cuda") and spec is None
                       and getattr(self.runner, "supports_async", False))
        self._inflight: List[_InFlight] = []
        self._n_sync_only = 0
        self._beams = BeamSearcher(self)
        self.spec = None
        if spec is not None:
            from rusteeze_b200.engine.spec_decode import SpecDecoder
            self.spec = SpecDecoder(self, spec)

    # ------------------------------------------------------------------ sizing
    def _profile_num_blocks(self) -> int:
        ec = self.config.engine
        bytes_per_block = self.model_config.kv_bytes_per_token(torch.finfo(self.kv_dtype).bits // 8) * BLOCK_SIZE
        bytes_per_block //= max(1, getattr(self.model.tp, "size", 1)) if self.model_config.num_key_value_heads >= \
            getattr(self.model.tp, "size", 1) else 1
        if not self.device.startswith("cuda"):
            return 64 if self.model_config.hidden_size <= 512 else 512
        free, total = torch.cuda.mem_get_info()
        used_by_others = total - free
        budget = total * ec.gpu_memory_utilization - used_by_others
        # activations / logits / graph pools headroom
        budget -= 4 * (1 << 30)
        # a separate draft model (speculative decoding): its weights, and one draft KV block per block
        from rusteeze_b200.engine.spec_decode import draft_memory
        d_w, d_blk = draft_memory(self.model_config, ec.speculative, torch.finfo(self.dtype).bits // 8, BLOCK_SIZE)
        budget -= d_w
        bytes_per_block += d_blk
        n = int(budget // bytes_per_block)
        if n < 16:
            raise RuntimeError(f"not enough GPU memory for the KV cache ({budget / 2**30:.1f} GiB left)")
        return n

    # ------------------------------------------------------------------ requests
    def add_request(self, request_id: Optional[str], prompt: Optional[str] = None,
                    params: Optional[SamplingParams] = None, prompt_token_ids: Optional[List[int]] = None,
                    arrival_time: Optional[float] = None, priority: int = 0) -> Request:
        params = params or SamplingParams()
        if prompt_token_ids is None:
            if prompt is None:
                raise InvalidRequestError("either prompt or prompt_token_ids is required")
            prompt_token_ids = self.tokenizer.encode(prompt)
        if not prompt_token_ids:
            raise InvalidRequestError("empty prompt")
        V = self.model_config.vocab_size
        if min(prompt_token_ids) < 0 or max(prompt_token_ids) >= V:
            raise InvalidRequestError(f"prompt token ids must be in [0, {V})")
        # token ids the sampler indexes logits with: out of range they would fail inside step()
        for what, ids in (("logit_bias", params.logit_bias.keys()), ("stop_token_ids", params.stop_token_ids)):
            if any(not 0 <= int(t) < V for t in ids):
                raise InvalidRequestError(f"{what} token ids must be in [0, {V})")
        if len(prompt_token_ids) >= self.max_model_len:
            raise ContextLengthExceededError(
                f"prompt has {len(prompt_token_ids)} tokens; the model context is {self.max_model_len}")
        guide = None
        if params.guided_decoding is not None:
            if params.use_beam_search:
                raise InvalidRequestError("beam search cannot be combined with guided decoding")
            from rusteeze_b200.engine.guided import Guide, fsm_for, guide_pattern, index_for
            try:
                fsm = fsm_for(guide_pattern(params.guided_decoding))
            except ValueError as e:
                raise InvalidRequestError(f"guided decoding: {e}", param="guided_decoding") from None
            guide = Guide(fsm, index_for(self.tokenizer, V), self.eos_ids)
        if params.use_beam_search:
            if self.spec is not None:
                raise InvalidRequestError("beam search cannot be combined with speculative decoding")
            if params.best_of > self.scheduler.cfg.max_num_seqs:
                raise InvalidRequestError(f"beam width {params.best_of} exceeds max_num_seqs "
                                          f"({self.scheduler.cfg.max_num_seqs}): the beams could never step together")
        rid = request_id or new_request_id("cmpl")
        if rid in self.requests:
            raise InvalidRequestError(f"duplicate request id {rid}")
        req = Request(rid, prompt, list(prompt_token_ids), params,
                      arrival_time if arrival_time is not None else time.monotonic(), priority)
        if params.seed is None:
            req.seed = int(self._rng.integers(0, 2 ** 62))
        else:
            req.seed = int(params.seed)
        if params.use_beam_search:
            self._beams.start(req)
        if guide is not None:
            req.seqs[0].guide = guide
        for s in req.seqs:
            self._register_seq(req, s)
            self.scheduler.add(s)
        req.async_ok = (Sampler.async_eligible(params) and params.n == 1 and params.best_of == 1)
        if not req.async_ok:
            self._n_sync_only += 1
        self.requests[rid] = req
        return req

    def _register_seq(self, req: Request, s: Sequence) -> None:
        if s.detok is None:
            s.detok = IncrementalDetokenizer(self.tokenizer, req.prompt_token_ids, req.params.skip_special_tokens)
        self.seq_to_request[s.seq_id] = req

    def abort_request(self, request_id: str) -> bool:
        req = self.requests.get(request_id)
        if req is None:
            return False
        for s in req.seqs:
            if not s.is_finished():
                self.scheduler.remove(s)
                self.bm.free(s.seq_id)
                s.status = RequestStatus.FINISHED_ABORTED
                s.finish_reason = "abort"
        req.forked = True
        self.stats_counters["requests_aborted"] += 1
        self._retire(req)
        return True

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished() or bool(self._inflight)

    def get_num_unfinished_requests(self) -> int:
        return len(self.requests)

    # ------------------------------------------------------------------ step
    def step(self) -> List[RequestOutput]:
        if self.spec is not None:
            return self.spec.step()
        if self._async:
            if self._n_sync_only == 0:
                return self._step_async()
            if self._inflight:          # a request needs host-side sampling state: drain, then go synchronous
                return self._drain_inflight()
        h0 = time.perf_counter()
        with nvtx_range("rz.step.schedule"):
            so = self.scheduler.schedule()
        if so.preempted:
            self._release_slots(so.preempted)
        outputs: List[RequestOutput] = []
        if so.is_empty():
            # nothing to run, but a swap-in or swap-out decided this step must still happen
            self.runner.apply_block_ops(so)
            return self._collect_ignored()
        rows, owners = self._sample_rows(so)
        t0 = time.monotonic()
        h1 = time.perf_counter()
        with nvtx_range("rz.step.execute"):
            res = self.runner.execute(so, self.bm, rows)
        h2 = time.perf_counter()
        now = time.monotonic()
        self.stats_counters["steps"] += 1
        touched = self._apply_results(so, res, owners, now)
        for obs in self.observers:
            obs(self, so, now - t0)
        outputs += self._emit(touched)
        outputs += self._collect_ignored()
        ph = self.phase_s
        ph["schedule"] += h1 - h0
        ph["postprocess"] += time.perf_counter() - h2
        return outputs

    def host_phase_seconds(self) -> Dict[str, float]:
        """Cumulative host seconds per step phase (schedule, prepare, enqueue,
        sample_wait = sampling incl. the wait for the GPU, postprocess)."""
        d = dict(self.phase_s)
        d.update(getattr(self.runner, "phase_s", {}))
        return d

    # ------------------------------------------------------------------ asynchronous scheduling
    def _step_async(self) -> List[RequestOutput]:
        """One pipelined step: schedule and enqueue step n+1 (decode inputs of
        sequences whose step-n token is still on the GPU are scattered from
        step n's sample tensor on the device), then wait for step n and apply
        its tokens while the GPU runs n+1.  Outputs lag one step; stop
        conditions found in step n's tokens discard the sequence's token of
        step n+1 (its KV write lands in blocks that are only reused by later
        steps, which the stream orders after it)."""
        h0 = time.perf_counter()
        with nvtx_range("rz.step.schedule"):
            so = self.scheduler.schedule()
        if so.preempted:
            self._release_slots(so.preempted)
        launched = False
        if so.is_empty():
            self.runner.apply_block_ops(so)        # block moves of a step with nothing to run
        else:
            prev = self._inflight[-1] if self._inflight else None
            for ss in so.scheduled:
                if ss.seq.pending:
                    ss.pend_row = prev.rows_of[ss.seq.seq_id]
            rows, owners = self._sample_rows(so)
            h1 = time.perf_counter()
            self.phase_s["schedule"] += h1 - h0
            with nvtx_range("rz.step.launch"):
                handle = self.runner.launch(so, self.bm, rows, prev.handle.tokens if prev is not None else None)
            rows_of: Dict[int, int] = {}
            i = 0
            for ss, k in owners:
                rows_of[ss.seq.seq_id] = i
                i += k
            for ss in so.scheduled:
                s = ss.seq
                if s.num_generated == 0 and s.pending == 0:
                    self.stats_counters["prompt_tokens"] += ss.num_new
                s.num_computed = ss.ctx + ss.num_new
                if ss.sample:
                    s.pending += 1
            self._inflight.append(_InFlight(so, handle, owners, rows_of, time.monotonic()))
            self.stats_counters["steps"] += 1
            launched = True
        outputs: List[RequestOutput] = []
        if len(self._inflight) > (1 if launched else 0):
            outputs = self._finish_oldest()
        return outputs + self._collect_ignored()

    def _finish_oldest(self) -> List[RequestOutput]:
        done = self._inflight.pop(0)
        res = self.runner.finish(done.handle)
        h2 = time.perf_counter()
        now = time.monotonic()
        touched, seen = [], set()
        i = 0
        for ss, k in done.owners:
            s = ss.seq
            req = s.request
            tok, lp = res.tokens[i], res.logprobs[i]
            i += k
            s.pending -= 1
            if s.is_finished() or req.request_id not in self.requests:
                continue                  # finished or aborted after this step was launched
            s.append_token(tok, None)
            if req.metrics.first_token_time is None:
                req.metrics.first_token_time = now
            req.metrics.last_token_time = now
            req.metrics.num_generated = max(req.metrics.num_generated, s.num_generated)
            self.stats_counters["generation_tokens"] += 1
            try:
                self._check_stop(s, tok)
            except Exception as e:  # noqa: BLE001 -- this request's host-side processing only
                self._fail_request(req, e)
            if id(req) not in seen:
                seen.add(id(req))
                touched.append(req)
        # publish the now-known full blocks to the prefix cache
        if self._prefix_caching:
            for ss in done.so.scheduled:
                s = ss.seq
                if not s.is_finished() and self.bm.has_seq(s.seq_id):
                    self.bm.commit(s.seq_id, s.tokens_np(), min(s.num_computed, len(s.token_ids)))
        for obs in self.observers:
            obs(self, done.so, now - done.t_launch)
        outputs = self._emit(touched)
        self.phase_s["postprocess"] += time.perf_counter() - h2
        return outputs

    def _emit(self, touched) -> List[RequestOutput]:
        """Outputs of the requests a step advanced: every step for streaming requests,
        only the last one for final-only requests; finished requests are retired."""
        outputs = []
        for req in touched:
            fin = req.is_finished()
            if fin or (req.stream and req.beam is None):
                outputs.append(req.to_output(delta=True))
            if fin:
                self._retire(req)
        return outputs

    def _drain_inflight(self) -> List[RequestOutput]:
        outs: List[RequestOutput] = []
        while self._inflight:
            outs += self._finish_oldest()
        return outs + self._collect_ignored()

    def _collect_ignored(self) -> List[RequestOutput]:
        outs = []
        if not self.scheduler.ignored:
            return outs
        ign, self.scheduler.ignored = self.scheduler.ignored, []
        for s in ign:
            req = s.request
            # ignored before its best_of samples were forked: there will be no children
            req.forked = True
            if req.request_id in self.requests and req.is_finished():
                outs.append(req.to_output(delta=True))
                self._retire(req)
        return outs

    def _sample_rows(self, so):
        rows: List[SampleRow] = []
        owners = []
        for ss in so.scheduled:
            if not ss.sample:
                continue
            s = ss.seq
            req = s.request
            p = req.params
            if req.beam is not None:
                rows.append(SampleRow(req.beam.row_params, None, None, req.seed, s.num_generated + s.pending,
                                      self.eos_ids, None, s, 0))
                owners.append((ss, 1))
                continue
            # token histories are read from the sequence only by rows that need them
            mask = s.guide.mask(allow_eos=not p.ignore_eos) if s.guide is not None else None
            for j in range(ss.num_samples):
                rows.append(SampleRow(p, None, None, req.seed + 7919 * (s.index + j), s.num_generated + s.pending,
                                      self.eos_ids, s.mirostat_mu, s, j))
                rows[-1].allowed = mask
            owners.append((ss, ss.num_samples))
        return rows, owners

    def _apply_results(self, so, res, owners, now: float):
        touched = []
        seen = set()
        # advance computed counters and publish full blocks to the prefix cache
        for ss in so.scheduled:
            s = ss.seq
            s.num_computed = ss.ctx + ss.num_new
            self.bm.commit(s.seq_id, s.tokens_np(), s.num_computed)
            if s.num_generated == 0:
                self.stats_counters["prompt_tokens"] += ss.num_new
        i = 0
        beams = {}
        failed = set()
        for ss, k in owners:
            s = ss.seq
            req = s.request
            i0, i = i, i + k
            if id(req) in failed:
                continue
            try:
                if req.params.prompt_logprobs is not None and req.prompt_lp is None and s.num_generated == 0:
                    req.prompt_lp = self._score_prompt(s, req.params.prompt_logprobs)
                if req.beam is not None:
                    beams.setdefault(id(req), (req, []))[1].append((s, ss, res.top_logprobs[i0]))
                    continue
                self._apply_samples(req, s, k, res, i0, now)
            except Exception as e:  # noqa: BLE001 -- this request's host-side processing only
                failed.add(id(req))
                self._fail_request(req, e)
            if id(req) not in seen:
                seen.add(id(req))
                touched.append(req)
        for key, (req, entries) in beams.items():
            if key in failed:
                continue
            try:
                self._beams.step(req, entries, now)
            except Exception as e:  # noqa: BLE001
                self._fail_request(req, e)
            if key not in seen:
                seen.add(key)
                touched.append(req)
        return touched

    def _apply_samples(self, req: Request, s: Sequence, k: int, res, i: int, now: float) -> None:
        """The k tokens sampled for sequence `s` (k > 1: the prompt row of a best_of
        request, whose samples fork the sequence)."""
        toks = res.tokens[i:i + k]
        lps = res.logprobs[i:i + k]
        tops = res.top_logprobs[i:i + k]
        mus = res.mirostat_mu[i:i + k]
        targets = [s]
        if k > 1:   # fork best_of - 1 children sharing the prompt's blocks (copy-on-write)
            for j in range(1, k):
                c = Sequence(req, req.prompt_token_ids, index=j)
                c.num_computed = s.num_computed
                c.num_cached = s.num_cached
                c.guide = s.guide.copy() if s.guide is not None else None
                self.bm.fork(s.seq_id, c.seq_id)
                req.seqs.append(c)
                self._register_seq(req, c)
                self.scheduler.add_running(c)
                targets.append(c)
            req.forked = True
        for t, tok, lp, top, mu in zip(targets, toks, lps, tops, mus):
            t.append_token(tok, lp, top)
            if mu is not None:
                t.mirostat_mu = mu
            if req.metrics.first_token_time is None:
                req.metrics.first_token_time = now
            req.metrics.last_token_time = now
            req.metrics.num_generated = max(req.metrics.num_generated, t.num_generated)
            self.stats_counters["generation_tokens"] += 1
            self._check_stop(t, tok)

    def _fail_request(self, req: Request, exc: BaseException) -> None:
        """A request's host-side processing (detokenisation, stop checks, guided decoding,
        beam search, prompt scoring) raised: that request ends, aborted, with the error as
        its stop reason, and the rest of the batch carries on.  Errors of the step itself
        (the forward, the sampler, a device fault) still fail the engine."""
        log.error("request %s failed in post-processing: %r", req.request_id, exc, exc_info=exc)
        for s in req.seqs:
            if not s.is_finished():
                self.scheduler.remove(s)
                self.bm.free(s.seq_id)
                s.status = RequestStatus.FINISHED_ABORTED
                s.finish_reason = "abort"
                s.stop_reason = f"error: {exc!r}"[:300]
        req.forked = True
        self.stats_counters["requests_failed"] = self.stats_counters.get("requests_failed", 0) + 1

    # ------------------------------------------------------------------ embeddings
    @torch.no_grad()
    def embed(self, inputs: List[List[int]], pooling: str = "last", normalize: bool = True) -> List[np.ndarray]:
        """Embeddings of token sequences: the model's final normalised hidden state of the
        last token (`last`, the pooling of decoder embedding models) or the mean over all
        tokens (`mean`), L2-normalised unless `normalize` is False.

        Each input is run between engine steps in blocks of its own: allocated under
        placeholder token ids that no prefix-cache block matches and never published, so
        an embedding neither reads nor rewrites the prefix cache.  Inputs longer than one
        step's token budget run in chunks, attending to the chunks before them."""
        if pooling not in ("last", "mean"):
            raise InvalidRequestError(f"pooling must be last or mean, got {pooling!r}", param="pooling")
        if self._inflight:
            raise RuntimeError("embed() runs between steps: drain the pipelined steps first")
        from rusteeze_b200.core.errors import ServiceUnavailableError
        from rusteeze_b200.engine.sequence import _seq_ids
        V = self.model_config.vocab_size
        runner = self.runner
        cap = getattr(runner, "max_tokens", None) or getattr(getattr(runner, "runner", None), "max_tokens", 512)
        if pooling == "mean" and self.model_config_tp() > 1:
            cap = min(cap, 512)           # every row's logits are computed (and dropped) at TP > 1
        out = []
        for toks in inputs:
            L = len(toks)
            if L == 0:
                raise InvalidRequestError("an embedding input must not be empty")
            if min(toks) < 0 or max(toks) >= V:
                raise InvalidRequestError(f"token ids must be in [0, {V})")
            if L > self.max_model_len:
                raise ContextLengthExceededError(f"input has {L} tokens; the model context is {self.max_model_len}")
            placeholder = np.full(L, -1, dtype=np.int64)
            if self.bm.blocks_needed_for_prompt(placeholder, L) > self.bm.num_free_gpu_blocks():
                raise ServiceUnavailableError("not enough free KV cache blocks for this input right now")
            sid = next(_seq_ids)
            arr = np.asarray(toks, dtype=np.int64)
            self.bm.allocate_prompt(sid, placeholder)
            try:
                self.bm.ensure_capacity(sid, L, 0)
                acc, vec, c0 = None, None, 0
                while c0 < L:
                    n = min(cap, L - c0)
                    rows = n if pooling == "mean" else 1
                    hs = runner.forward_arrays(self.bm, [sid], [c0], [n], arr[c0:c0 + n], rows, 0,
                                               hidden=True).float()
                    if pooling == "mean":
                        part = hs.sum(0)
                        acc = part if acc is None else acc + part
                    elif c0 + n == L:
                        vec = hs[-1]
                    c0 += n
            finally:
                self.bm.free(sid)
            if pooling == "mean":
                vec = acc / L
            if normalize:
                vec = vec / vec.norm().clamp_min(1e-12)
            out.append(vec.cpu().numpy())
        return out

    def model_config_tp(self) -> int:
        return int(getattr(getattr(self.model, "tp", None), "size", 1) or 1)

    @torch.no_grad()
    def _score_prompt(self, s: Sequence, k: int) -> List[Optional[Dict[int, float]]]:
        """Prompt logprobs (`prompt_logprobs` = k): one extra forward over the prompt, whose
        KV is already in the cache, in chunks that fit the runner's staging buffers; the
        logits at position j - 1 score prompt token j.  The batched step computes logits
        for sampled positions only, so scoring runs apart from it, once per request."""
        P = s.prompt_len
        toks = np.asarray(s.token_ids[:P], dtype=np.int64)
        runner = self.runner
        cap = getattr(runner, "max_tokens", None) or getattr(getattr(runner, "runner", None), "max_tokens", P)
        out: List[Optional[Dict[int, float]]] = [None]
        c0 = 0
        while c0 < P - 1:
            n = min(cap, P - c0)
            logits = runner.forward_arrays(self.bm, [s.seq_id], [c0], [n], toks[c0:c0 + n], n, 0)
            lsm = torch.log_softmax(logits.float(), -1).cpu()
            for r in range(n):
                j = c0 + r + 1
                if j >= P:
                    break
                d: Dict[int, float] = {}
                if k:
                    v, ix = lsm[r].topk(min(k, lsm.shape[1]))
                    d = dict(zip(ix.tolist(), v.tolist()))
                d[int(toks[j])] = float(lsm[r, toks[j]])
                out.append(d)
            c0 += n
        return out

    def _check_stop(self, s: Sequence, tok: int) -> None:
        req = s.request
        p = req.params
        if req.defer_text or s.detok is None:
            delta = ""
        else:
            delta = s.detok.step(tok)
            s.detok_n += 1
            s.output_text += delta
        reason = None
        n = s.num_generated
        if s.guide is not None:
            s.guide.advance(tok)
        if n >= p.min_tokens:
            if not p.ignore_eos and tok in self.eos_ids:
                reason = "stop"
                s.stop_reason = None
            elif tok in p.stop_token_ids:
                reason = "stop"
                s.stop_reason = tok
            elif p.stop:
                for st in p.stop:
                    pos = s.output_text.find(st, max(0, len(s.output_text) - len(delta) - len(st)))
                    if pos >= 0:
                        s.output_text = s.output_text[:pos + (len(st) if p.include_stop_str_in_output else 0)]
                        reason = "stop"
                        s.stop_reason = st
                        break
        if reason is None and ((p.max_tokens is not None and n >= p.max_tokens)
                               or len(s.token_ids) >= self.max_model_len):
            reason = "length"
        if reason is None and s.guide is not None and (
                ((p.ignore_eos or not self.eos_ids) and s.guide.complete) or s.guide.stuck()):
            reason = "stop"               # complete with no EOS to come, or no token can continue it
        if reason is not None:
            s.finish_reason = reason
            s.status = RequestStatus.FINISHED_STOPPED if reason == "stop" else RequestStatus.FINISHED_LENGTH
            self.scheduler.remove(s)
            self.bm.free(s.seq_id)

    def _release_slots(self, seqs) -> None:
        sm = self._sampler
        if sm is not None:
            for s in seqs:
                sm.release(s.seq_id)

    def _retire(self, req: Request) -> None:
        import time as _t
        self._release_slots(req.seqs)
        if req.request_id in self.requests:
            if not getattr(req, "async_ok", True):
                self._n_sync_only -= 1
            req.metrics.finished_time = _t.monotonic()
            del self.requests[req.request_id]
            for s in req.seqs:
                self.seq_to_request.pop(s.seq_id, None)
            self.stats_counters["requests_finished"] += 1

    # ------------------------------------------------------------------ recovery
    def recover_from_worker_failure(self, executor, num_gpu_blocks: int) -> int:
        """A tensor-parallel worker died and the group was restarted (the launcher's
        `recover`): the KV cache is gone.  Steps in flight never completed, so their samples
        are dropped; every running or swapped sequence is reset for recompute and queued
        ahead of the waiting prompts in its old order, with a fresh block manager and the
        new executor.  Returns the number of sequences re-queued."""
        from collections import deque
        for fl in self._inflight:
            for ss, _k in fl.owners:
                ss.seq.pending = max(0, ss.seq.pending - 1)
        self._inflight = []
        live = [s for s in list(self.scheduler.running) + list(self.scheduler.swapped) if not s.is_finished()]
        waiting = [s for s in self.scheduler.waiting if not s.is_finished()]
        ec = self.config.engine
        num_cpu_blocks = swap_blocks(ec, self.model_config, self.dtype, self.device)
        self.bm = make_block_manager(BLOCK_SIZE, num_gpu_blocks, num_cpu_blocks, ec.enable_prefix_caching)
        n_pre = self.scheduler.num_preemptions
        self.scheduler = Scheduler(self.sched_cfg, self.bm)
        self.scheduler.num_preemptions = n_pre + len(live)
        for s in live:
            s.reset_for_recompute()
            s.pending = 0
        for s in waiting:
            if s.num_computed:
                s.reset_for_recompute()
        self.scheduler.waiting = deque(live + waiting)
        self.runner = executor
        self._sampler = getattr(executor, "sampler", None)
        if self._sampler is not None and self.device.startswith("cuda"):
            self._sampler.max_slots = ec.max_num_seqs + 64
        if self.device.startswith("cuda") and not ec.enforce_eager and hasattr(self.runner, "capture_graphs"):
            from rusteeze_b200.engine.model_runner import decode_graph_buckets
            mx = min(ec.cuda_graph_max_batch or ec.max_num_seqs, ec.max_num_seqs)
            self.runner.capture_graphs(decode_graph_buckets(mx))
        self.stats_counters["worker_recoveries"] = self.stats_counters.get("worker_recoveries", 0) + 1
        log.warning("worker group replaced: %d sequences re-queued for recompute", len(live))
        return len(live)

    # ------------------------------------------------------------------ stats
    def stats(self) -> dict:
        d = dict(self.stats_counters)
        d.update(num_waiting=self.scheduler.num_waiting, num_running=self.scheduler.num_running,
                 num_swapped=self.scheduler.num_swapped, num_preemptions=self.scheduler.num_preemptions,
                 kv_cache_usage=self.bm.gpu_usage(), num_gpu_blocks=self.bm.num_gpu_blocks)
        d.update({f"block_{k}": v for k, v in self.bm.stats().items()})
        return d


class LLM:
    """Offline batch API: `LLM(...).generate(prompts, SamplingParams(...))`, `chat(messages)`
    (rendered with the model's chat template, as the chat endpoint renders them) and
    `embed(texts)`."""

    def __init__(self, model: Optional[str] = None, *, preset: Optional[str] = None,
                 config: Optional[Config] = None, **engine_kw):
        from rusteeze_b200.config.config import Config as _C
        cfg = config or _C()
        if model is not None:
            if os.path.isdir(model):
                cfg.model.path = model
            else:
                cfg.model.preset = model
        if preset is not None:
            cfg.model.preset = preset
        for k, v in engine_kw.items():
            for sec in (cfg.engine, cfg.model):
                if hasattr(sec, k):
                    setattr(sec, k, v)
                    break
            else:
                raise TypeError(f"unknown option {k}")
        self.engine = LLMEngine(cfg)

    def generate(self, prompts: Union[None, str, List[str]] = None,
                 sampling_params: Optional[Union[SamplingParams, List[SamplingParams]]] = None,
                 prompt_token_ids: Optional[List[List[int]]] = None,
                 use_tqdm: bool = False) -> List[RequestOutput]:
        if isinstance(prompts, str):
            prompts = [prompts]
        n = len(prompts) if prompts is not None else len(prompt_token_ids)
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params or SamplingParams()] * n
        # offline batches read only the finished outputs
        sampling_params = [sp if sp.output_kind == "final_only" else sp.clone(output_kind="final_only")
                           for sp in sampling_params]
        ids = []
        for i in range(n):
            req = self.engine.add_request(
                None, prompts[i] if prompts is not None else None, sampling_params[i],
                prompt_token_ids[i] if prompt_token_ids is not None else None)
            ids.append(req.request_id)
        done: Dict[str, RequestOutput] = {}
        while self.engine.has_unfinished_requests():
            for out in self.engine.step():
                if out.finished:
                    done[out.request_id] = out
        return [done[i] for i in ids]

    @property
    def tokenizer(self):
        return self.engine.tokenizer

    def chat(self, messages, sampling_params: Optional[SamplingParams] = None, tools: Optional[List[Dict]] = None,
             chat_template: Optional[str] = None, add_generation_prompt: bool = True) -> List[RequestOutput]:
        """One conversation (a list of {role, content} messages) or a list of them."""
        from rusteeze_b200.tokenizer.chat_template import ChatTemplate
        convs = [messages] if messages and isinstance(messages[0], dict) else list(messages)
        eng = self.engine
        cfg = eng.config.model
        tmpl = (ChatTemplate(jinja=chat_template) if chat_template else
                ChatTemplate.for_model(cfg.path or eng.model_name, eng.tokenizer, cfg.chat_template))
        ids = []
        for conv in convs:
            text = tmpl.apply(conv, add_generation_prompt=add_generation_prompt, tools=tools)
            ids.append(eng.tokenizer.encode(text, add_special_tokens=False) or eng.tokenizer.encode(text))
        return self.generate(None, sampling_params, prompt_token_ids=ids)

    def embed(self, inputs: Union[str, List[str], List[List[int]]], pooling: str = "last",
              normalize: bool = True) -> List[np.ndarray]:
        """Embeddings of texts (tokenised with the model's tokenizer) or token id lists."""
        if isinstance(inputs, str):
            inputs = [inputs]
        lists = [self.engine.tokenizer.encode(x) if isinstance(x, str) else list(x) for x in inputs]
        return self.engine.embed(lists, pooling, normalize)

