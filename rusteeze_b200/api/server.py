"""OpenAI-compatible HTTP server.

Routes (crates/rusteeze-api/src/routes.rs:19-43): POST /v1/chat/completions
(streaming dispatch on `stream`), GET /v1/models, /health, /health/live,
/health/ready, /metrics, /version -- plus POST /v1/completions, which the
reference documents (crates/rusteeze-api/src/lib.rs:8) but never routes.
Chat prompts are rendered with the model's chat template (the reference
joins "role: content" lines, handlers.rs:222-229).  `stop`, `n`,
`best_of`, beam search, logprobs and `stream_options.include_usage` are honoured
(the reference ignores stop and n, handlers.rs:232-245).  SSE framing follows
handlers.rs:143-182: a role chunk, content deltas, a finish chunk, then
`data: [DONE]`.

Tool calling (`tools`, `tool_choice`: declared in crates/rusteeze-core/src/request.rs:91-95,
never read by the reference's handlers) renders the tools into the prompt; `required` or a
named function constrains the reply to one JSON call by guided decoding; `auto` returns a
call when the reply is one.

The engine runs in its own thread behind `AsyncLLMEngine`; handlers only
await per-request output queues.
"""
from __future__ import annotations

import json
import time
import uuid
from typing import AsyncIterator, List, Optional

from fastapi import FastAPI, Request
from fastapi.middleware.cors import CORSMiddleware
from fastapi.middleware.gzip import GZipMiddleware
from fastapi.responses import JSONResponse, PlainTextResponse, Response, StreamingResponse

from rusteeze_b200 import __version__
from rusteeze_b200.api import schemas as S
from rusteeze_b200.api.middleware import (AuthMiddleware, BodyLimitMiddleware, RateLimitMiddleware, RequestIdMiddleware,
                                          SlidingWindowLimiter, TimeoutMiddleware, error_response)
from rusteeze_b200.core.errors import InvalidRequestError, RusteezeError
from rusteeze_b200.core.sampling_params import EarlyStoppingMode, GuidedDecodingParams, SamplingParams
from rusteeze_b200.metrics.registry import CONTENT_TYPE, EngineMetrics
from rusteeze_b200.tokenizer.chat_template import ChatTemplate


def _guided(req) -> Optional[GuidedDecodingParams]:
    """The request's structured-output constraint, if any."""
    rf = req.response_format or {}
    t = rf.get("type") if isinstance(rf, dict) else None
    if t not in (None, "text", "json_object", "json_schema"):
        raise InvalidRequestError(f"response_format type {t!r} is not supported", param="response_format")
    g = GuidedDecodingParams()
    if t == "json_object":
        g.json_object = True
    elif t == "json_schema":
        js = rf.get("json_schema") or {}
        schema = js.get("schema", js) if isinstance(js, dict) else None
        if not isinstance(schema, dict):
            raise InvalidRequestError("response_format json_schema needs a schema object", param="response_format")
        g.json_schema = schema
    if req.guided_json is not None:
        g.json_schema = json.loads(req.guided_json) if isinstance(req.guided_json, str) else req.guided_json
    if req.guided_regex is not None:
        g.regex = req.guided_regex
    if req.guided_choice is not None:
        g.choice = list(req.guided_choice)
    if g.json_schema is None and g.regex is None and not g.choice and not g.json_object:
        return None
    return g


def _tool_setup(req):
    """(tools to render, function definitions, mode, JSON schema that forces a call or
    None).  mode: "none" (no tools, or tool_choice none), "auto" (the reply may be a call,
    parsed afterwards), "forced" (tool_choice required or a named function: the reply is
    constrained to {"name": ..., "arguments": ...} by guided decoding)."""
    tools = req.tools or []
    choice = req.tool_choice
    if not tools:
        if choice not in (None, "none", "auto"):
            raise InvalidRequestError("tool_choice needs tools", param="tool_choice")
        return None, [], "none", None
    fns = []
    for t in tools:
        f = t.get("function") if isinstance(t, dict) else None
        if not isinstance(t, dict) or t.get("type", "function") != "function" or not isinstance(f, dict) \
                or not f.get("name"):
            raise InvalidRequestError("each tool must be {type: function, function: {name, parameters}}",
                                      param="tools")
        fns.append(f)
    if choice in (None, "auto"):
        return tools, fns, "auto", None
    if choice == "none":
        return None, fns, "none", None
    if choice == "required":
        chosen = fns
    elif isinstance(choice, dict) and choice.get("type") == "function":
        name = (choice.get("function") or {}).get("name")
        chosen = [f for f in fns if f["name"] == name]
        if not chosen:
            raise InvalidRequestError(f"tool_choice names an unknown function {name!r}", param="tool_choice")
    else:
        raise InvalidRequestError("tool_choice must be none, auto, required or {type: function, function: {name}}",
                                  param="tool_choice")
    alts = [{"type": "object", "properties": {"name": {"const": f["name"]},
                                              "arguments": f.get("parameters") or {"type": "object"}},
             "required": ["name", "arguments"]} for f in chosen]
    return tools, fns, "forced", (alts[0] if len(alts) == 1 else {"anyOf": alts})


def _parse_tool_call(text: str, fns) -> Optional[dict]:
    """A reply that is exactly one JSON call of a known function, as an OpenAI tool call."""
    t = text.strip()
    if not t.startswith("{"):
        return None
    try:
        d = json.loads(t)
    except ValueError:
        return None
    if not isinstance(d, dict):
        return None
    args = d.get("arguments", d.get("parameters"))
    if d.get("name") not in {f["name"] for f in fns} or not isinstance(args, dict):
        return None
    return {"id": "call_" + uuid.uuid4().hex[:24], "type": "function",
            "function": {"name": d["name"], "arguments": json.dumps(args)}}


def _sampling_params(req, defaults, max_tokens_default: int, logprobs: Optional[int]) -> SamplingParams:
    stop = req.stop if isinstance(req.stop, list) else ([req.stop] if req.stop else [])
    mt = getattr(req, "max_completion_tokens", None) or req.max_tokens or max_tokens_default
    beam = req.use_beam_search
    # beam search is deterministic: unset temperature / top_p / top_k take its values,
    # not the server's sampling defaults
    es = req.early_stopping
    return SamplingParams(
        n=req.n, best_of=req.best_of or req.n, max_tokens=mt,
        temperature=req.temperature if req.temperature is not None else (0.0 if beam else defaults.temperature),
        top_p=req.top_p if req.top_p is not None else (1.0 if beam else defaults.top_p),
        top_k=req.top_k if req.top_k is not None else (-1 if beam else defaults.top_k),
        use_beam_search=beam, length_penalty=req.length_penalty, guided_decoding=_guided(req),
        early_stopping=EarlyStoppingMode(es if isinstance(es, str) else ("true" if es else "false")),
        min_p=req.min_p or 0.0,
        presence_penalty=req.presence_penalty or 0.0, frequency_penalty=req.frequency_penalty or 0.0,
        repetition_penalty=req.repetition_penalty if req.repetition_penalty is not None
        else defaults.repetition_penalty,
        stop=stop, stop_token_ids=req.stop_token_ids or [], seed=req.seed,
        logit_bias={int(k): v for k, v in (req.logit_bias or {}).items()},
        logprobs=logprobs, ignore_eos=req.ignore_eos, min_tokens=req.min_tokens,
        skip_special_tokens=req.skip_special_tokens,
        include_stop_str_in_output=req.include_stop_str_in_output,
        # a non-streaming response is built from the final output only
        output_kind="delta" if getattr(req, "stream", False) else "final_only")


def _sse(obj) -> str:
    if isinstance(obj, str):
        return f"data: {obj}\n\n"
    return "data: " + obj.model_dump_json(exclude_none=True) + "\n\n"


def create_app(async_engine, config=None, metrics: Optional[EngineMetrics] = None) -> FastAPI:
    from rusteeze_b200.config.config import Config
    cfg = config or Config()
    eng = async_engine.engine
    model_name = cfg.model.name or getattr(eng, "model_name", "model")
    metrics = metrics or EngineMetrics(model_name=model_name)
    if metrics.on_step not in eng.observers:
        eng.observers.append(metrics.on_step)
    template = ChatTemplate.for_model(model_name if not cfg.model.path else cfg.model.path, eng.tokenizer,
                                      cfg.model.chat_template)
    defaults = cfg.engine.sampling
    started = time.time()

    app = FastAPI(title="rusteeze_b200", version=__version__)
    app.state.engine = async_engine
    app.state.metrics = metrics
    sc = cfg.server
    app.add_middleware(TimeoutMiddleware, timeout_s=sc.timeout_seconds)
    limiter = None
    if sc.rate_limit is not None and sc.rate_limit.enabled:
        rl = sc.rate_limit
        limiter = SlidingWindowLimiter(rl.requests_per_minute, rl.burst, rl.requests_per_day,
                                       tokens_per_minute=rl.tokens_per_minute, tokens_per_day=rl.tokens_per_day)
        app.add_middleware(RateLimitMiddleware, limiter=limiter, by=rl.by)
    app.state.rate_limiter = limiter
    app.add_middleware(AuthMiddleware, api_key=sc.api_key)
    if sc.compression:
        app.add_middleware(GZipMiddleware, minimum_size=1024)
    if sc.cors.enabled:
        app.add_middleware(CORSMiddleware, allow_origins=sc.cors.allowed_origins,
                           allow_methods=sc.cors.allowed_methods, allow_headers=sc.cors.allowed_headers,
                           max_age=sc.cors.max_age)
    app.add_middleware(RequestIdMiddleware, log_requests=cfg.logging.request_logging)
    app.add_middleware(BodyLimitMiddleware, max_bytes=sc.max_body_bytes)

    @app.exception_handler(RusteezeError)
    async def _err(_request: Request, exc: RusteezeError):
        metrics.errors.labels(exc.code).inc()
        return error_response(exc)

    @app.exception_handler(ValueError)
    async def _verr(_request: Request, exc: ValueError):
        return error_response(InvalidRequestError(str(exc)))

    def _charge(key: Optional[str], final) -> None:
        """Token limits: a generation's prompt + completion tokens go to its client's key."""
        if limiter is not None and key is not None and final is not None:
            limiter.charge(key, len(final.prompt_token_ids) + sum(len(c.token_ids) for c in final.outputs))

    def _check_model(name: str) -> None:
        if name and name != model_name and not cfg.model.path == name:
            from rusteeze_b200.core.errors import NotFoundError
            raise NotFoundError(f"model {name!r} not found; this server serves {model_name!r}")

    # ------------------------------------------------------------------ completions
    @app.post("/v1/completions")
    async def completions(req: S.CompletionRequest, request: Request):
        _check_model(req.model)
        prompts: List = []
        p = req.prompt
        if isinstance(p, str):
            prompts = [(p, None)]
        elif p and isinstance(p[0], int):
            prompts = [(None, list(p))]
        elif p and isinstance(p[0], list):
            prompts = [(None, list(x)) for x in p]
        else:
            prompts = [(x, None) for x in p]
        if not prompts:
            raise InvalidRequestError("prompt must not be empty")
        sp = _sampling_params(req, defaults, 16, req.logprobs)
        if req.echo and req.logprobs is not None:
            sp.prompt_logprobs = req.logprobs        # echoed prompt tokens carry logprobs too
        metrics.on_request_params(sp)
        rid = "cmpl-" + uuid.uuid4().hex
        key = getattr(request.state, "rate_key", None)
        if req.stream:
            return StreamingResponse(_stream_completion(rid, prompts, sp, req, key), media_type="text/event-stream")
        choices, usage = [], S.Usage()
        for pi, (text, ids) in enumerate(prompts):
            final = None
            async for out in async_engine.generate(text, sp, f"{rid}-{pi}", ids, priority=req.priority):
                final = out
            metrics.on_request_finished(final, "completions")
            _charge(key, final)
            usage.prompt_tokens += len(final.prompt_token_ids)
            for c in final.outputs:
                usage.completion_tokens += len(c.token_ids)
                t = ((final.prompt or eng.tokenizer.decode(final.prompt_token_ids)) if req.echo else "") + c.text
                echo_lp = (final.prompt_token_ids, final.prompt_logprobs) if (
                    req.echo and final.prompt_logprobs is not None) else None
                choices.append(S.CompletionChoice(index=pi * sp.n + c.index, text=t, finish_reason=c.finish_reason,
                                                  logprobs=_cmpl_logprobs(eng.tokenizer, c, echo_lp)
                                                  if req.logprobs is not None else None))
        usage.total_tokens = usage.prompt_tokens + usage.completion_tokens
        return S.CompletionResponse(id=rid, model=model_name, choices=choices, usage=usage)

    async def _stream_completion(rid, prompts, sp, req, key) -> AsyncIterator[str]:
        usage = S.Usage()
        try:
            for pi, (text, ids) in enumerate(prompts):
                final = None
                agen = async_engine.generate(text, sp, f"{rid}-{pi}", ids, priority=req.priority)
                completed = False
                sent, offs = {}, {}                # tokens and text characters already sent, per output
                try:
                    async for out in agen:
                        final = out
                        for c, delta in zip(out.outputs, out.delta_text):
                            lp = None
                            if req.logprobs is not None and len(c.token_ids) > sent.get(c.index, 0):
                                lp = _cmpl_logprobs(eng.tokenizer, _TokSlice(c, sent.get(c.index, 0)),
                                                    offset=offs.get(c.index, 0))
                                sent[c.index] = len(c.token_ids)
                                offs[c.index] = lp.text_offset[-1] + len(lp.tokens[-1])
                            if delta or c.finish_reason or lp is not None:
                                chunk = S.CompletionResponse(
                                    id=rid, model=model_name, usage=S.Usage(),
                                    choices=[S.CompletionChoice(index=pi * sp.n + c.index, text=delta,
                                                                finish_reason=c.finish_reason, logprobs=lp)])
                                yield "data: " + chunk.model_dump_json(exclude={"usage"}, exclude_none=True) + "\n\n"
                    completed = True
                finally:
                    await agen.aclose()           # a stream closed early aborts its request now, not at GC
                    _charge(key, final)
                    if not completed:
                        metrics.on_request_finished(final, "completions", status="aborted")
                metrics.on_request_finished(final, "completions")
                usage.prompt_tokens += len(final.prompt_token_ids)
                usage.completion_tokens += sum(len(c.token_ids) for c in final.outputs)
            if req.stream_options and req.stream_options.include_usage:
                usage.total_tokens = usage.prompt_tokens + usage.completion_tokens
                yield "data: " + json.dumps({"id": rid, "object": "text_completion", "model": model_name,
                                             "choices": [], "usage": usage.model_dump()}) + "\n\n"
        except RusteezeError as e:
            yield "data: " + json.dumps(e.to_openai()) + "\n\n"
        yield _sse("[DONE]")

    # ------------------------------------------------------------------ chat
    @app.post("/v1/chat/completions")
    async def chat(req: S.ChatCompletionRequest, request: Request):
        _check_model(req.model)
        msgs = [m.model_dump() for m in req.messages]
        tools, fns, tool_mode, call_schema = _tool_setup(req)
        if req.chat_template and not sc.trust_request_chat_template:
            raise InvalidRequestError("a per-request chat_template is disabled on this server "
                                      "(server.trust_request_chat_template)", param="chat_template")
        tmpl = template if not req.chat_template else ChatTemplate(jinja=req.chat_template)
        try:
            prompt = tmpl.apply(msgs, add_generation_prompt=req.add_generation_prompt, tools=tools)
        except RusteezeError:
            raise
        except Exception as e:  # noqa: BLE001 -- template syntax errors, raise_exception(), bad messages
            raise InvalidRequestError(f"chat template could not render these messages: {e}",
                                      param="messages") from None
        ids = eng.tokenizer.encode(prompt, add_special_tokens=False) or eng.tokenizer.encode(prompt)
        lp = (req.top_logprobs or 0) if req.logprobs else None
        sp = _sampling_params(req, defaults, defaults.max_tokens, lp)
        if call_schema is not None:
            if sp.guided_decoding is not None:
                raise InvalidRequestError("tool_choice required / named cannot be combined with response_format "
                                          "or guided decoding", param="tool_choice")
            sp.guided_decoding = GuidedDecodingParams(json_schema=call_schema)
        metrics.on_request_params(sp)
        rid = "chatcmpl-" + uuid.uuid4().hex
        key = getattr(request.state, "rate_key", None)
        if req.stream:
            return StreamingResponse(_stream_chat(rid, ids, sp, req, key, tool_mode, fns),
                                     media_type="text/event-stream")
        final = None
        async for out in async_engine.generate(None, sp, rid, ids, priority=req.priority):
            final = out
        metrics.on_request_finished(final, "chat")
        _charge(key, final)
        choices = []
        for c in final.outputs:
            call = _parse_tool_call(c.text, fns) if tool_mode != "none" and c.finish_reason == "stop" else None
            msg = (S.ChatMessage(role="assistant", content=None, tool_calls=[call]) if call is not None
                   else S.ChatMessage(role="assistant", content=c.text))
            choices.append(S.ChatChoice(index=c.index, message=msg,
                                        finish_reason="tool_calls" if call is not None else c.finish_reason,
                                        logprobs=_chat_logprobs(eng.tokenizer, c) if req.logprobs else None))
        n_out = sum(len(c.token_ids) for c in final.outputs)
        return S.ChatCompletionResponse(id=rid, model=model_name, choices=choices,
                                        usage=S.Usage(prompt_tokens=len(ids), completion_tokens=n_out,
                                                      total_tokens=len(ids) + n_out))

    async def _stream_chat(rid, ids, sp, req, key, tool_mode="none", fns=()) -> AsyncIterator[str]:
        for i in range(sp.n):
            yield _sse(S.ChatCompletionChunk(id=rid, model=model_name, choices=[
                S.ChatChunkChoice(index=i, delta=S.ChatDelta(role="assistant", content=""))]))
        final = None
        agen = async_engine.generate(None, sp, rid, ids, priority=req.priority)
        completed = False
        try:
            try:
                # with tools, a reply that opens with "{" is held back until it is known
                # whether it is a call (sent as one tool_calls delta) or text
                held: dict = {}
                passthrough: dict = {}
                sent: dict = {}                   # tokens whose logprobs were sent, per output
                async for out in agen:
                    final = out
                    for c, delta in zip(out.outputs, out.delta_text):
                        i = c.index
                        if tool_mode != "none" and not passthrough.get(i):
                            held[i] = held.get(i, "") + delta
                            lead = held[i].lstrip()
                            if lead and not lead.startswith("{") and tool_mode == "auto":
                                passthrough[i] = True
                                delta, held[i] = held[i], ""
                            else:
                                delta = ""
                        lp = None
                        if req.logprobs and not held.get(i) and len(c.token_ids) > sent.get(i, 0):
                            lp = _chat_logprobs(eng.tokenizer, _TokSlice(c, sent.get(i, 0)))
                            sent[i] = len(c.token_ids)
                        if delta or lp is not None:
                            yield _sse(S.ChatCompletionChunk(id=rid, model=model_name, choices=[
                                S.ChatChunkChoice(index=i, delta=S.ChatDelta(content=delta), logprobs=lp)]))
                        if c.finish_reason:
                            reason = c.finish_reason
                            if held.get(i):
                                call = _parse_tool_call(held[i], fns) if reason == "stop" else None
                                if call is not None:
                                    reason = "tool_calls"
                                    d = S.ChatDelta(tool_calls=[{"index": 0, **call}])
                                else:
                                    d = S.ChatDelta(content=held[i])
                                held[i] = ""
                                yield _sse(S.ChatCompletionChunk(id=rid, model=model_name, choices=[
                                    S.ChatChunkChoice(index=i, delta=d)]))
                            yield _sse(S.ChatCompletionChunk(id=rid, model=model_name, choices=[
                                S.ChatChunkChoice(index=i, delta=S.ChatDelta(), finish_reason=reason)]))
                completed = True
            finally:
                await agen.aclose()               # a stream closed early aborts its request now, not at GC
                _charge(key, final)
                if not completed:
                    metrics.on_request_finished(final, "chat", status="aborted")
            metrics.on_request_finished(final, "chat")
            if req.stream_options and req.stream_options.include_usage and final is not None:
                n_out = sum(len(c.token_ids) for c in final.outputs)
                yield _sse(S.ChatCompletionChunk(id=rid, model=model_name, choices=[], usage=S.Usage(
                    prompt_tokens=len(ids), completion_tokens=n_out, total_tokens=len(ids) + n_out)))
        except RusteezeError as e:
            yield "data: " + json.dumps(e.to_openai()) + "\n\n"
        yield _sse("[DONE]")

    # ------------------------------------------------------------------ embeddings
    @app.post("/v1/embeddings")
    async def embeddings(req: S.EmbeddingRequest, request: Request):
        """The final hidden state of each input's last token (or the mean over its tokens),
        L2-normalised; `dimensions` keeps the first d components (renormalised);
        `encoding_format` base64 is the little-endian float32 bytes."""
        _check_model(req.model)
        inp = req.input
        if isinstance(inp, str):
            lists = [eng.tokenizer.encode(inp)]
        elif inp and all(isinstance(x, str) for x in inp):
            lists = [eng.tokenizer.encode(x) for x in inp]
        elif inp and all(isinstance(x, int) for x in inp):
            lists = [list(inp)]
        else:
            lists = [list(x) for x in inp]
        if not lists or any(len(x) == 0 for x in lists):
            raise InvalidRequestError("input must not be empty", param="input")
        vecs = await async_engine.embed(lists, req.pooling, req.normalize)
        import base64
        import numpy as np
        data = []
        for i, v in enumerate(vecs):
            v = np.asarray(v, dtype=np.float32)
            if req.dimensions is not None:
                if not 1 <= req.dimensions <= v.shape[0]:
                    raise InvalidRequestError(f"dimensions must be in [1, {v.shape[0]}]", param="dimensions")
                v = v[:req.dimensions]
                if req.normalize:
                    v = v / max(float(np.linalg.norm(v)), 1e-12)
            emb = (base64.b64encode(v.astype("<f4").tobytes()).decode() if req.encoding_format == "base64"
                   else v.tolist())
            data.append(S.EmbeddingData(embedding=emb, index=i))
        n = sum(len(x) for x in lists)
        key = getattr(request.state, "rate_key", None)
        if limiter is not None and key is not None:
            limiter.charge(key, n)
        return S.EmbeddingResponse(data=data, model=model_name,
                                   usage=S.EmbeddingUsage(prompt_tokens=n, total_tokens=n))

    # ------------------------------------------------------------------ tokenizer
    @app.post("/tokenize")
    async def tokenize(req: S.TokenizeRequest):
        """Token ids of a prompt (or of chat messages as the chat endpoint renders them),
        with the model's context length, so a client can count before it sends."""
        _check_model(req.model)
        if (req.prompt is None) == (req.messages is None):
            raise InvalidRequestError("give exactly one of prompt or messages")
        if req.messages is not None:
            text = template.apply([m.model_dump() for m in req.messages],
                                  add_generation_prompt=req.add_generation_prompt)
            ids = eng.tokenizer.encode(text, add_special_tokens=False) or eng.tokenizer.encode(text)
        else:
            ids = eng.tokenizer.encode(req.prompt, add_special_tokens=req.add_special_tokens)
        return {"tokens": ids, "count": len(ids), "max_model_len": getattr(eng, "max_model_len", None)}

    @app.post("/detokenize")
    async def detokenize(req: S.DetokenizeRequest):
        _check_model(req.model)
        V = eng.model_config.vocab_size
        if any(not 0 <= t < V for t in req.tokens):
            raise InvalidRequestError(f"token ids must be in [0, {V})", param="tokens")
        return {"prompt": eng.tokenizer.decode(req.tokens, req.skip_special_tokens)}

    # ------------------------------------------------------------------ misc
    @app.get("/v1/models")
    async def models():
        return S.ModelList(data=[S.ModelCard(id=model_name, max_model_len=getattr(eng, "max_model_len", None))])

    @app.get("/health")
    async def health():
        st = async_engine.stats()
        gpu = 0.0
        try:
            import torch
            if torch.cuda.is_available():
                free, total = torch.cuda.mem_get_info()
                gpu = 1.0 - free / total
        except Exception:  # noqa: BLE001
            pass
        body = S.HealthResponse(status="healthy" if async_engine.is_ready else "unhealthy", version=__version__,
                                uptime_seconds=int(time.time() - started),
                                requests_processed=st.get("requests_processed", 0),
                                waiting_requests=st.get("num_waiting", 0), running_requests=st.get("num_running", 0),
                                gpu_memory_usage=gpu, kv_cache_usage=st.get("kv_cache_usage", 0.0))
        return JSONResponse(body.model_dump(), status_code=200 if async_engine.is_ready else 503)

    @app.get("/health/live")
    async def live():
        return PlainTextResponse("OK")

    @app.get("/health/ready")
    async def ready():
        if async_engine.is_ready:
            return PlainTextResponse("READY")
        return PlainTextResponse("NOT READY", status_code=503)

    @app.get(cfg.metrics.path if cfg.metrics.enabled else "/metrics")
    async def metrics_endpoint():
        return Response(metrics.export(), media_type=CONTENT_TYPE)

    @app.get("/version")
    async def version():
        import torch
        return {"version": __version__, "name": "rusteeze_b200", "torch": torch.__version__,
                "cuda": torch.version.cuda, "arch": "sm_100a"}

    return app


class _TokSlice:
    """The tokens (and their logprob tables) of one output not yet sent on a stream."""
    __slots__ = ("token_ids", "logprobs")

    def __init__(self, c, start: int):
        self.token_ids = c.token_ids[start:]
        self.logprobs = (c.logprobs or [])[start:]


def _cmpl_logprobs(tok, c, prompt=None, offset: int = 0) -> S.CompletionLogProbs:
    """OpenAI completion logprobs; with `echo`, the prompt's tokens come first (the first
    one without a logprob, as it has no context).  `offset`: text offset of the first token
    (streams send later tokens in later chunks)."""
    lp = S.CompletionLogProbs()
    off = offset
    if prompt is not None:
        ids, plp = prompt
        for tid, d in zip(ids, plp):
            s = tok.decode([tid])
            lp.tokens.append(s)
            lp.token_logprobs.append(None if d is None else d.get(tid))
            lp.top_logprobs.append(None if d is None else {tok.decode([k]): v for k, v in d.items()})
            lp.text_offset.append(off)
            off += len(s)
    for tid, d in zip(c.token_ids, c.logprobs or []):
        s = tok.decode([tid])
        lp.tokens.append(s)
        lp.token_logprobs.append(d.get(tid))
        lp.top_logprobs.append({tok.decode([k]): v for k, v in d.items()})
        lp.text_offset.append(off)
        off += len(s)
    return lp


def _chat_logprobs(tok, c) -> S.ChatLogProbs:
    content = []
    for tid, d in zip(c.token_ids, c.logprobs or []):
        s = tok.decode([tid])
        content.append(S.TokenLogProb(token=s, logprob=d.get(tid, 0.0), bytes=list(s.encode()),
                                      top_logprobs=[S.TopLogProb(token=t, logprob=v, bytes=list(t.encode()))
                                                    for t, v in ((tok.decode([k]), v) for k, v in d.items()
                                                                 if k != tid)]))
    return S.ChatLogProbs(content=content)


def serve(config, engine=None, host: Optional[str] = None, port: Optional[int] = None) -> None:
    """Builds the engine (unless given; D replicas behind a router when
    model.data_parallel_size = D > 1), starts the engine thread(s) and runs uvicorn
    with graceful SIGINT/SIGTERM shutdown (crates/rusteeze-api/src/server.rs:304-330).
    TLS is real when cert/key are configured (the reference falls back to
    plaintext, server.rs:185-192)."""
    import uvicorn
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    from rusteeze_b200.engine.llm_engine import LLMEngine
    if engine is None and config.model.data_parallel_size > 1:
        from rusteeze_b200.engine.dp_engine import ReplicatedAsyncEngine
        ae = ReplicatedAsyncEngine.from_config(config).start()
    else:
        eng = engine or LLMEngine(config)
        ae = AsyncLLMEngine(eng, request_timeout_s=config.engine.request_timeout_seconds).start()
    metrics = EngineMetrics(model_name=config.model.served_name())
    app = create_app(ae, config, metrics)
    if config.server.metrics_port:
        from rusteeze_b200.metrics.exporter import start_exporter
        start_exporter(metrics, config.server.metrics_port)
    pusher = None
    pg = config.metrics.push_gateway
    if pg is not None and pg.url:
        from rusteeze_b200.metrics.exporter import PushGatewayPusher
        pusher = PushGatewayPusher(metrics, pg.url, pg.job, pg.instance, pg.interval_seconds).start()
    tls = config.server.tls
    kw = {}
    if tls is not None and tls.cert_path:
        kw.update(ssl_certfile=tls.cert_path, ssl_keyfile=tls.key_path)
    uv = uvicorn.Config(app, host=host or config.server.host, port=port or config.server.port,
                        log_level=config.logging.level.lower().replace("warn", "warning"),
                        timeout_keep_alive=int(config.server.keep_alive_seconds),
                        limit_concurrency=config.server.max_connections, **kw)
    server = uvicorn.Server(uv)
    try:
        server.run()
    finally:
        ae.shutdown()
        if pusher is not None:
            pusher.stop()


def serve_from_env() -> None:
    """RUSTEEZE_HOST / RUSTEEZE_PORT / RUSTEEZE_API_KEY / RUSTEEZE_MODEL... (server.rs:333-370)."""
    from rusteeze_b200.config.loader import load_config
    serve(load_config())
