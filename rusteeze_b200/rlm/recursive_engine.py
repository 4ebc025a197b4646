"""Recursive Language Model (RLM) engine: host orchestration over the LLM engine.

Algorithm (crates/rusteeze-engine/src/recursive_engine.rs:265-491): the
prompt is stored as a variable, never placed in the model context; prompts
above `auto_decompose_threshold` characters (100K) are pre-chunked; then up
to `max_iterations` turns of: context = system prompt + constant-size
metadata -> model -> parse one operation -> execute -> sub-calls -> repeat,
until FINAL / FINAL_VAR.  Cost is tracked per 1K input/output tokens.

Differences by design:
  * BATCH_SUBCALL / map sub-calls are submitted to the engine TOGETHER
    (`InferenceModel.infer_batch`), so they run as one continuous batch on
    the GPU; the reference runs them one after another (:401-442).
  * Sub-calls go through `RecursiveScheduler` (depth, pending and per-level
    limits, timeouts, cascading cancel); the reference creates it and
    ignores it (:283).
  * A sub-call whose text is itself longer than the threshold recurses into
    a child RLM (depth-limited) instead of being truncated to ctx*3 chars.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Protocol, Tuple

from rusteeze_b200.rlm.prompt_env import (OP_PATTERN, EnvLimits, ExecResult, PromptEnvironment, adaptive_chunk,
                                          parse_model_output)
from rusteeze_b200.rlm.recursive_scheduler import RecursiveScheduler, SchedulerLimits

SYSTEM_PROMPT = """You are operating a REPL over a long prompt stored in variable __prompt__.
You never see the whole prompt; you see metadata and the results of your operations.
Respond with exactly one operation per turn, on its own line:
  PEEK(start_byte, end_byte)          read part of the prompt
  SEARCH(pattern)                     regex search in the prompt
  DECOMPOSE(chunk_chars, overlap)     split the prompt into __chunks__
  SUBCALL(text, instruction)          ask a sub-model about literal text
  SUBCALL_VAR(var, instruction)       ask a sub-model about a variable
  BATCH_SUBCALL(list_var, instruction) ask about every item of a list (in parallel)
  SET_VAR(name, value) / GET_VAR(name)
  TRANSFORM(src, dst, op)             op: split(d) join(d) filter(k) sort count truncate(n) grep(re)
                                      map_subcall(instruction) reduce_subcall(instruction)
  FINAL(answer) / FINAL_VAR(name)     finish
"""


@dataclass
class InferenceResult:
    text: str
    prompt_tokens: int = 0
    completion_tokens: int = 0


class InferenceModel(Protocol):
    def infer(self, prompt: str, max_tokens: int) -> InferenceResult: ...

    def infer_batch(self, prompts: List[str], max_tokens: int) -> List[InferenceResult]: ...


@dataclass
class RLMConfig:
    max_iterations: int = 50
    max_depth: int = 3
    max_subcalls: int = 1000
    session_timeout_s: float = 600.0
    root_max_tokens: int = 4096
    subcall_max_tokens: int = 2048
    auto_decompose: bool = True
    auto_decompose_threshold: int = 100_000
    auto_chunk_chars: int = 8000
    auto_chunk_overlap: int = 200
    cost_per_1k_input: float = 0.001
    cost_per_1k_output: float = 0.003
    per_level_concurrency: int = 16
    # constrain the orchestrator's turns to one operation line (`OP_PATTERN`, guided
    # decoding) when the model supports it: a turn can then always be parsed
    constrain_ops: bool = True


@dataclass
class RLMStats:
    iterations: int = 0
    subcalls: int = 0
    batch_subcalls: int = 0
    max_depth_reached: int = 0
    prompt_tokens: int = 0
    completion_tokens: int = 0
    auto_decomposed: bool = False
    elapsed_s: float = 0.0

    @property
    def cost(self) -> float:
        return 0.0


@dataclass
class RLMResponse:
    text: str
    terminated: bool
    stats: RLMStats
    cost_usd: float
    trace: List[str] = field(default_factory=list)


class RecursiveEngine:
    def __init__(self, model: InferenceModel, config: Optional[RLMConfig] = None):
        self.model = model
        self.config = config or RLMConfig()
        self.global_stats = {"sessions": 0, "iterations": 0, "subcalls": 0, "cost_usd": 0.0}

    # ------------------------------------------------------------------ public
    def process(self, prompt: str, instruction: str = "", depth: int = 0,
                scheduler: Optional[RecursiveScheduler] = None, parent_call: int = 0) -> RLMResponse:
        cfg = self.config
        t0 = time.monotonic()
        limits = EnvLimits(max_iterations=cfg.max_iterations, max_depth=cfg.max_depth,
                           max_subcalls=cfg.max_subcalls, session_timeout_s=cfg.session_timeout_s)
        env = PromptEnvironment(prompt, limits, depth=depth)
        sched = scheduler or RecursiveScheduler(SchedulerLimits(max_depth=cfg.max_depth,
                                                                max_pending=cfg.max_subcalls,
                                                                per_level_concurrency=cfg.per_level_concurrency))
        stats = RLMStats(max_depth_reached=depth)
        trace: List[str] = []
        if cfg.auto_decompose and len(prompt) > cfg.auto_decompose_threshold:
            env.store.set(env.CHUNKS_VAR, adaptive_chunk(prompt, cfg.auto_chunk_chars, cfg.auto_chunk_overlap))
            stats.auto_decomposed = True
        task = f"\nTask: {instruction}\n" if instruction else ""
        last = env.initial_metadata()
        for it in range(cfg.max_iterations):
            if env.timed_out():
                trace.append("session timeout")
                break
            env.iteration = it + 1
            stats.iterations += 1
            context = SYSTEM_PROMPT + task + "\n" + (last if it == 0 else env.iteration_metadata(last))
            kw = ({"pattern": OP_PATTERN} if cfg.constrain_ops and getattr(self.model, "supports_pattern", False)
                  else {})
            r = self.model.infer(context, cfg.root_max_tokens, **kw)
            stats.prompt_tokens += r.prompt_tokens
            stats.completion_tokens += r.completion_tokens
            op = parse_model_output(r.text)
            trace.append(f"{op.kind}{op.args!r}"[:200])
            res = env.execute(op)
            if res.error:
                last = "ERROR: " + res.error
                continue
            if res.subcalls:
                last = self._run_subcalls(env, res, sched, parent_call, stats, depth)
            else:
                last = res.stdout
            if env.is_terminated():
                break
        out = env.store.final_value()
        terminated = out is not None
        if out is None:
            out = last
        stats.elapsed_s = time.monotonic() - t0
        cost = (stats.prompt_tokens / 1000.0) * cfg.cost_per_1k_input + \
               (stats.completion_tokens / 1000.0) * cfg.cost_per_1k_output
        if depth == 0:
            self.global_stats["sessions"] += 1
            self.global_stats["iterations"] += stats.iterations
            self.global_stats["subcalls"] += stats.subcalls
            self.global_stats["cost_usd"] += cost
        return RLMResponse(out, terminated, stats, cost, trace)

    # ------------------------------------------------------------------ sub-calls
    def _run_subcalls(self, env: PromptEnvironment, res: ExecResult, sched: RecursiveScheduler, parent: int,
                      stats: RLMStats, depth: int) -> str:
        cfg = self.config
        subs = res.subcalls
        try:
            ids = sched.spawn_batch(parent, [(s.prompt, s.instruction) for s in subs])
        except (RecursionError, RuntimeError) as e:
            return f"ERROR: {e}"
        env.subcalls_made += len(subs)
        stats.subcalls += len(subs)
        stats.max_depth_reached = max(stats.max_depth_reached, depth + 1)
        if len(subs) > 1:
            stats.batch_subcalls += 1
        results: List[Optional[str]] = [None] * len(subs)
        # long sub-prompts recurse (depth permitting); the rest go to the model together
        direct: List[int] = []
        for i, (s, cid) in enumerate(zip(subs, ids)):
            if len(s.prompt) > cfg.auto_decompose_threshold and depth + 1 < cfg.max_depth:
                sched.start(cid)
                child = self.process(s.prompt, s.instruction, depth + 1, sched, cid)
                stats.prompt_tokens += child.stats.prompt_tokens
                stats.completion_tokens += child.stats.completion_tokens
                stats.max_depth_reached = max(stats.max_depth_reached, child.stats.max_depth_reached)
                results[i] = child.text
                sched.complete(cid, child.text)
            else:
                direct.append(i)
        pending = list(direct)
        while pending:
            ready_ids = {n.call_id for n in sched.ready()}
            wave = [i for i in pending if ids[i] in ready_ids] or pending[:1]
            for i in wave:
                sched.start(ids[i])
            prompts = [f"{subs[i].instruction}\n\n{subs[i].prompt}" for i in wave]
            outs = self.model.infer_batch(prompts, cfg.subcall_max_tokens)
            for i, o in zip(wave, outs):
                stats.prompt_tokens += o.prompt_tokens
                stats.completion_tokens += o.completion_tokens
                results[i] = o.text
                sched.complete(ids[i], o.text)
            pending = [i for i in pending if i not in wave]
        if res.batch_target:
            env.store_batch_results(res.batch_target, [r or "" for r in results])
            return f"{len(results)} sub-call results stored in {res.batch_target}"
        for s, r in zip(subs, results):
            env.store_subcall_result(s, r or "")
        tgt = subs[0].target_var
        return f"sub-call result stored in {tgt}: {(results[0] or '')[:500]}"


# ----------------------------------------------------------------------------- adapters
class EngineInferenceModel:
    """InferenceModel over an LLMEngine: `infer_batch` submits every prompt
    at once so the engine batches them (continuous batching on the GPU)."""

    def __init__(self, engine, temperature: float = 0.0, max_context_tokens: Optional[int] = None):
        self.engine = engine
        self.temperature = temperature
        self.max_ctx = max_context_tokens or (engine.max_model_len - 16)
        self._n = 0

    def _clip(self, ids: List[int], max_tokens: int) -> Tuple[List[int], int]:
        room = self.max_ctx - max(16, min(max_tokens, self.max_ctx // 2))
        if len(ids) > room:
            ids = ids[:room // 2] + ids[-(room - room // 2):]
        return ids, min(max_tokens, self.max_ctx - len(ids))

    supports_pattern = True

    def infer_batch(self, prompts: List[str], max_tokens: int,
                    pattern: Optional[str] = None) -> List[InferenceResult]:
        from rusteeze_b200.core.sampling_params import GuidedDecodingParams, SamplingParams
        guided = GuidedDecodingParams(regex=pattern) if pattern else None
        rids = []
        for p in prompts:
            ids, mt = self._clip(self.engine.tokenizer.encode(p), max_tokens)
            self._n += 1
            rid = f"rlm-{self._n}"
            self.engine.add_request(rid, None, SamplingParams(temperature=self.temperature, max_tokens=max(1, mt),
                                                              guided_decoding=guided), ids)
            rids.append(rid)
        done: Dict[str, object] = {}
        while any(r not in done for r in rids):
            for o in self.engine.step():
                if o.finished:
                    done[o.request_id] = o
        out = []
        for r in rids:
            o = done[r]
            out.append(InferenceResult(o.outputs[0].text, len(o.prompt_token_ids), len(o.outputs[0].token_ids)))
        return out

    def infer(self, prompt: str, max_tokens: int, pattern: Optional[str] = None) -> InferenceResult:
        return self.infer_batch([prompt], max_tokens, pattern)[0]


class MockInferenceModel:
    """Keyword -> response fake for tests (the reference's MockInferenceModel,
    recursive_engine.rs:905-959): the first rule whose keyword occurs in the
    prompt wins; `auto_resolve` makes the root FINAL after N turns."""

    def __init__(self, rules: Optional[List[Tuple[str, str]]] = None, default: str = "THINK",
                 auto_resolve: Optional[int] = None):
        self.rules = rules or []
        self.default = default
        self.auto_resolve = auto_resolve
        self.calls: List[str] = []
        self.batch_sizes: List[int] = []

    def infer(self, prompt: str, max_tokens: int) -> InferenceResult:
        self.calls.append(prompt)
        if self.auto_resolve is not None and prompt.startswith(SYSTEM_PROMPT):
            turns = sum(1 for c in self.calls if c.startswith(SYSTEM_PROMPT))
            if turns >= self.auto_resolve:
                return InferenceResult("FINAL(auto-resolved)", len(prompt) // 4, 4)
        for kw, resp in self.rules:
            if kw in prompt:
                r = resp(prompt) if callable(resp) else resp
                return InferenceResult(r, len(prompt) // 4, len(r) // 4)
        return InferenceResult(self.default, len(prompt) // 4, 1)

    def infer_batch(self, prompts: List[str], max_tokens: int) -> List[InferenceResult]:
        self.batch_sizes.append(len(prompts))
        return [self.infer(p, max_tokens) for p in prompts]
