"""API tier: OpenAI schema, SSE framing, health/metrics/models/version,
auth and rate limiting -- against the real engine on the tiny CPU model."""
import json

import pytest
from fastapi.testclient import TestClient

from rusteeze_b200.config.config import Config, RateLimitConfig
from rusteeze_b200.engine.async_engine import AsyncLLMEngine
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.api.server import create_app


def _cfg(api_key=None, rate=None):
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 128
    cfg.engine.max_num_seqs = 8
    cfg.engine.max_num_batched_tokens = 512
    cfg.engine.enable_chunked_prefill = True
    cfg.server.api_key = api_key
    cfg.logging.request_logging = False
    if rate:
        cfg.server.rate_limit = RateLimitConfig(enabled=True, requests_per_minute=rate, burst=0)
    return cfg


@pytest.fixture(scope="module")
def engine():
    return LLMEngine(_cfg())


def _client(engine, **kw):
    cfg = _cfg(**kw)
    ae = AsyncLLMEngine(engine).start()
    return TestClient(create_app(ae, cfg)), ae


def test_completions_basic(engine):
    c, ae = _client(engine)
    r = c.post("/v1/completions", json={"model": "tiny-llama", "prompt": "hello world", "max_tokens": 5,
                                        "temperature": 0, "ignore_eos": True})
    assert r.status_code == 200, r.text
    d = r.json()
    assert d["object"] == "text_completion" and d["id"].startswith("cmpl-")
    assert d["usage"]["completion_tokens"] == 5
    assert d["choices"][0]["finish_reason"] == "length"
    assert r.headers.get("x-request-id")
    ae.shutdown()


def test_completions_token_ids_n_and_logprobs(engine):
    c, ae = _client(engine)
    r = c.post("/v1/completions", json={"prompt": [[5, 6, 7, 8], [9, 10, 11]], "max_tokens": 3, "n": 2,
                                        "temperature": 0.8, "seed": 3, "logprobs": 2, "ignore_eos": True})
    assert r.status_code == 200, r.text
    d = r.json()
    assert len(d["choices"]) == 4
    assert d["usage"]["prompt_tokens"] == 7
    lp = d["choices"][0]["logprobs"]
    assert len(lp["token_logprobs"]) == 3 and all(v <= 0 for v in lp["token_logprobs"])
    ae.shutdown()


def test_completions_stream_sse(engine):
    c, ae = _client(engine)
    with c.stream("POST", "/v1/completions", json={"prompt": "abc", "max_tokens": 4, "stream": True,
                                                   "temperature": 0, "ignore_eos": True,
                                                   "stream_options": {"include_usage": True}}) as r:
        lines = [ln for ln in r.iter_lines() if ln]
    assert lines[-1] == "data: [DONE]"
    payloads = [json.loads(ln[6:]) for ln in lines[:-1]]
    assert payloads[-1]["usage"]["completion_tokens"] == 4
    assert any(p.get("choices") and p["choices"][0].get("finish_reason") == "length" for p in payloads)
    ae.shutdown()


def test_chat_and_chat_stream(engine):
    c, ae = _client(engine)
    body = {"model": "tiny-llama", "messages": [{"role": "system", "content": "be brief"},
                                                 {"role": "user", "content": "hi"}],
            "max_tokens": 4, "temperature": 0, "ignore_eos": True}
    r = c.post("/v1/chat/completions", json=body)
    assert r.status_code == 200, r.text
    d = r.json()
    assert d["object"] == "chat.completion"
    assert d["choices"][0]["message"]["role"] == "assistant"
    assert d["usage"]["completion_tokens"] == 4
    with c.stream("POST", "/v1/chat/completions", json={**body, "stream": True}) as rs:
        lines = [ln for ln in rs.iter_lines() if ln]
    assert lines[-1] == "data: [DONE]"
    first = json.loads(lines[0][6:])
    assert first["object"] == "chat.completion.chunk"
    assert first["choices"][0]["delta"]["role"] == "assistant"
    fins = [json.loads(x[6:]) for x in lines[:-1]]
    assert fins[-1]["choices"][0]["finish_reason"] == "length"
    ae.shutdown()


def test_stop_strings_and_validation(engine):
    c, ae = _client(engine)
    r = c.post("/v1/completions", json={"prompt": "x", "max_tokens": 4, "temperature": -1})
    assert r.status_code == 400 and r.json()["error"]["type"] == "invalid_request_error"
    r = c.post("/v1/completions", json={"prompt": "x", "max_tokens": 4, "model": "other"})
    assert r.status_code == 404
    ae.shutdown()


def test_health_models_version_metrics(engine):
    c, ae = _client(engine)
    assert c.get("/health/live").text == "OK"
    assert c.get("/health/ready").status_code == 200
    h = c.get("/health").json()
    assert h["status"] == "healthy"
    m = c.get("/v1/models").json()
    assert m["data"][0]["id"] == "tiny-llama"
    assert c.get("/version").json()["arch"] == "sm_100a"
    c.post("/v1/completions", json={"prompt": "metrics", "max_tokens": 2, "ignore_eos": True})
    text = c.get("/metrics").text
    assert "rusteeze_inference_generation_tokens_total" in text
    assert "rusteeze_inference_time_to_first_token_seconds_bucket" in text
    ae.shutdown()


def test_auth(engine):
    c, ae = _client(engine, api_key="sekret")
    assert c.post("/v1/completions", json={"prompt": "a", "max_tokens": 1}).status_code == 401
    r = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 1},
               headers={"Authorization": "Bearer sekret"})
    assert r.status_code == 200
    assert c.get("/health/live").status_code == 200      # probes stay open
    ae.shutdown()


def test_rate_limit_headers(engine):
    c, ae = _client(engine, rate=2)
    codes = []
    for _ in range(3):
        r = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 1})
        codes.append(r.status_code)
        assert "x-ratelimit-limit" in r.headers
    assert codes == [200, 200, 429]
    ae.shutdown()


def test_token_limiter_windows():
    """Token charges age out of the minute and day windows; a key at its limit waits until
    enough of its charges have aged out; keys are independent."""
    from rusteeze_b200.api.middleware import SlidingWindowLimiter
    lim = SlidingWindowLimiter(1000, 0, tokens_per_minute=100, tokens_per_day=250)
    assert lim.check("a", now=0.0)[0]
    lim.charge("a", 60, now=1.0)
    assert lim.check("a", now=2.0)[0] and lim.tokens_remaining("a", now=2.0) == 40
    lim.charge("a", 50, now=3.0)                       # 110 >= 100: the next request waits
    ok, _, _, wait = lim.check("a", now=4.0)
    assert not ok and wait == 57.0                     # the 60-token charge leaves at t = 61
    assert lim.check("b", now=4.0)[0]                  # another key is not affected
    assert lim.check("a", now=61.5)[0]                 # 50 tokens left in the minute window
    lim.charge("a", 90, now=62.0)
    lim.charge("a", 60, now=130.0)                     # day: 60 + 50 + 90 + 60 = 260 >= 250
    ok, _, _, wait = lim.check("a", now=131.0)
    assert not ok and wait == 86400.0 - 130.0          # until the first charge (t = 1) leaves the day
    assert lim.check("a", now=86402.0)[0]


def test_tokens_per_minute_limit_through_the_api(engine):
    cfg = _cfg()
    cfg.server.rate_limit = RateLimitConfig(enabled=True, requests_per_minute=100, burst=0, tokens_per_minute=30)
    ae = AsyncLLMEngine(engine).start()
    try:
        c = TestClient(create_app(ae, cfg))
        body = {"prompt": [1, 2, 3, 4, 5, 6, 7, 8, 9, 10], "max_tokens": 8, "ignore_eos": True}
        r = c.post("/v1/completions", json=body, headers={"x-api-key": "alice"})
        assert r.status_code == 200 and r.json()["usage"]["total_tokens"] == 18
        assert r.headers["x-ratelimit-limit-tokens"] == "30"
        r = c.post("/v1/completions", json=dict(body, stream=True), headers={"x-api-key": "alice"})
        assert r.status_code == 200                    # 18 < 30: admitted; charged 18 more when it ends
        r = c.post("/v1/completions", json=body, headers={"x-api-key": "alice"})
        assert r.status_code == 429 and int(r.headers["retry-after"]) >= 1
        assert r.headers["x-ratelimit-remaining-tokens"] == "0"
        r = c.post("/v1/chat/completions", headers={"x-api-key": "bob"},
                   json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4})
        assert r.status_code == 200                    # another key has its own budget
    finally:
        ae.shutdown()


def test_streamed_logprobs_equal_the_non_streamed_ones(engine):
    """Each stream chunk carries the logprobs of the tokens it adds; joined, they are the
    non-streamed response's (completions with absolute text offsets, and chat)."""
    c, ae = _client(engine)
    try:
        body = {"prompt": [7, 8, 9, 10], "max_tokens": 6, "temperature": 0, "ignore_eos": True, "logprobs": 2}
        full = c.post("/v1/completions", json=body).json()["choices"][0]["logprobs"]
        r = c.post("/v1/completions", json=dict(body, stream=True))
        joined = {"tokens": [], "token_logprobs": [], "top_logprobs": [], "text_offset": []}
        for ln in r.text.splitlines():
            if ln.startswith("data: {"):
                for ch in json.loads(ln[6:])["choices"]:
                    for k in joined:
                        joined[k] += (ch.get("logprobs") or {}).get(k, [])
        assert joined == full
        msgs = [{"role": "user", "content": "hi"}]
        chat = {"messages": msgs, "max_tokens": 5, "temperature": 0, "ignore_eos": True, "logprobs": True,
                "top_logprobs": 2}
        full = c.post("/v1/chat/completions", json=chat).json()["choices"][0]["logprobs"]["content"]
        r = c.post("/v1/chat/completions", json=dict(chat, stream=True))
        got = []
        for ln in r.text.splitlines():
            if ln.startswith("data: {"):
                for ch in json.loads(ln[6:])["choices"]:
                    got += (ch.get("logprobs") or {}).get("content") or []
        assert got == full and len(got) == 5
    finally:
        ae.shutdown()


def test_tokenize_and_detokenize(engine):
    c, ae = _client(engine)
    try:
        r = c.post("/tokenize", json={"prompt": "hello"})
        d = r.json()
        assert d["tokens"] == engine.tokenizer.encode("hello") and d["count"] == len(d["tokens"])
        assert d["max_model_len"] == engine.max_model_len
        r = c.post("/tokenize", json={"prompt": "hello", "add_special_tokens": False})
        assert r.json()["tokens"] == engine.tokenizer.encode("hello", add_special_tokens=False)
        msgs = [{"role": "user", "content": "hi"}]
        n_chat = c.post("/tokenize", json={"messages": msgs}).json()["count"]
        done = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 1}).json()
        assert n_chat == done["usage"]["prompt_tokens"]
        r = c.post("/detokenize", json={"tokens": engine.tokenizer.encode("hello", add_special_tokens=False)})
        assert r.json()["prompt"] == "hello"
        assert c.post("/detokenize", json={"tokens": [10 ** 9]}).status_code == 400
        assert c.post("/tokenize", json={}).status_code == 400
    finally:
        ae.shutdown()


def test_ready_reports_unhealthy_after_engine_failure():
    cfg = _cfg()
    eng = LLMEngine(cfg)
    ae = AsyncLLMEngine(eng).start()

    def boom():
        raise RuntimeError("injected step failure")

    eng.step = boom
    c = TestClient(create_app(ae, cfg))
    r = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 2})
    assert r.status_code == 503
    assert c.get("/health/ready").status_code == 503
    ae.shutdown()
