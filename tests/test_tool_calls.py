"""Tool calling on /v1/chat/completions: a named or `required` tool_choice yields a
`tool_calls` reply whose arguments satisfy the function's parameter schema (guided decoding
forces it, so random weights suffice), in one response or one stream delta; `auto` returns
a call only when the reply is one; tool definitions, earlier calls and tool results reach
the prompt; bad tool requests are refused."""
import json

import pytest
from fastapi.testclient import TestClient

from rusteeze_b200.api.server import _parse_tool_call, create_app
from rusteeze_b200.config.config import Config
from rusteeze_b200.engine.async_engine import AsyncLLMEngine
from rusteeze_b200.engine.llm_engine import LLMEngine

WEATHER = {"type": "function", "function": {
    "name": "get_weather", "description": "Weather in a city",
    "parameters": {"type": "object", "properties": {"city": {"type": "string", "maxLength": 8},
                                                    "days": {"type": "integer"}},
                   "required": ["city", "days"]}}}
TIME = {"type": "function", "function": {
    "name": "get_time", "parameters": {"type": "object", "properties": {"tz": {"enum": ["utc", "cet"]}},
                                       "required": ["tz"]}}}
# random weights: lean on the closing characters so every constrained reply ends early
BIAS = {str(ord(ch) + 3): b for ch, b in (("}", 5.0), ('"', 3.0), (",", 1.0))}


@pytest.fixture(scope="module")
def client():
    cfg = Config()
    cfg.model.preset, cfg.model.device, cfg.model.dtype = "tiny-llama", "cpu", "float32"
    cfg.engine.num_gpu_blocks = 256
    cfg.engine.max_num_seqs = 8
    cfg.engine.max_num_batched_tokens = 1024
    cfg.engine.enable_chunked_prefill = True
    cfg.logging.request_logging = False
    ae = AsyncLLMEngine(LLMEngine(cfg)).start()
    yield TestClient(create_app(ae, cfg))
    ae.shutdown()


def _chat(client, **kw):
    body = {"messages": [{"role": "user", "content": "weather in Oslo for 2 days?"}], "max_tokens": 120,
            "temperature": 0.8, "seed": 7, "logit_bias": BIAS}
    body.update(kw)
    return client.post("/v1/chat/completions", json=body)


def _check_weather_args(call):
    assert call["type"] == "function" and call["id"].startswith("call_")
    assert call["function"]["name"] == "get_weather"
    args = json.loads(call["function"]["arguments"])
    assert set(args) == {"city", "days"} and isinstance(args["city"], str) and len(args["city"]) <= 8
    assert type(args["days"]) is int


def test_named_tool_choice_returns_a_valid_call(client):
    for seed in range(3):
        r = _chat(client, tools=[WEATHER, TIME], seed=seed,
                  tool_choice={"type": "function", "function": {"name": "get_weather"}})
        assert r.status_code == 200, r.text
        ch = r.json()["choices"][0]
        assert ch["finish_reason"] == "tool_calls" and ch["message"]["content"] is None
        _check_weather_args(ch["message"]["tool_calls"][0])


def test_required_tool_choice_picks_one_of_the_tools(client):
    names = set()
    for seed in range(4):
        r = _chat(client, tools=[WEATHER, TIME], tool_choice="required", seed=seed)
        ch = r.json()["choices"][0]
        assert ch["finish_reason"] == "tool_calls", ch
        call = ch["message"]["tool_calls"][0]
        names.add(call["function"]["name"])
        if call["function"]["name"] == "get_time":
            assert json.loads(call["function"]["arguments"])["tz"] in ("utc", "cet")
        else:
            _check_weather_args(call)
    assert names <= {"get_weather", "get_time"}


def test_streamed_forced_call_is_one_tool_calls_delta(client):
    r = _chat(client, tools=[WEATHER], tool_choice="required", stream=True)
    chunks = [json.loads(ln[6:]) for ln in r.text.splitlines() if ln.startswith("data: {")]
    deltas = [c["choices"][0] for c in chunks if c["choices"]]
    calls = [d["delta"]["tool_calls"] for d in deltas if d["delta"].get("tool_calls")]
    assert len(calls) == 1 and calls[0][0]["index"] == 0
    _check_weather_args(calls[0][0])
    assert not any(d["delta"].get("content") for d in deltas)
    assert deltas[-1]["finish_reason"] == "tool_calls"


def test_auto_and_none_return_text_from_a_model_that_does_not_call(client):
    for choice in ("auto", "none"):
        r = _chat(client, tools=[WEATHER], tool_choice=choice, logit_bias={}, max_tokens=8)
        ch = r.json()["choices"][0]
        assert ch["finish_reason"] != "tool_calls" and ch["message"].get("tool_calls") is None
        assert isinstance(ch["message"]["content"], str)
    r = _chat(client, tools=[WEATHER], tool_choice="auto", logit_bias={}, max_tokens=8, stream=True)
    text = "".join(json.loads(ln[6:])["choices"][0]["delta"].get("content") or ""
                   for ln in r.text.splitlines() if ln.startswith("data: {") and json.loads(ln[6:])["choices"])
    plain = _chat(client, tools=[WEATHER], tool_choice="auto", logit_bias={}, max_tokens=8)
    assert text == plain.json()["choices"][0]["message"]["content"]


def test_parse_tool_call():
    fns = [WEATHER["function"]]
    c = _parse_tool_call(' {"name": "get_weather", "arguments": {"city": "x", "days": 1}} ', fns)
    assert c["function"] == {"name": "get_weather", "arguments": json.dumps({"city": "x", "days": 1})}
    assert _parse_tool_call('{"name": "get_weather", "parameters": {"city": "x"}}', fns) is not None
    for t in ('{"name": "other", "arguments": {}}', "hello", '{"name": "get_weather"}', "[1]", '{"name": '):
        assert _parse_tool_call(t, fns) is None


def test_multi_turn_with_tool_results(client):
    msgs = [{"role": "user", "content": "weather?"},
            {"role": "assistant", "content": None, "tool_calls": [
                {"id": "call_1", "type": "function",
                 "function": {"name": "get_weather", "arguments": '{"city": "Oslo", "days": 1}'}}]},
            {"role": "tool", "tool_call_id": "call_1", "content": "sunny"}]
    r = _chat(client, messages=msgs, tools=[WEATHER], max_tokens=4, logit_bias={})
    assert r.status_code == 200, r.text


@pytest.mark.parametrize("kw", [
    {"tool_choice": "required"},                                           # no tools
    {"tools": [{"type": "retrieval"}]},
    {"tools": [WEATHER], "tool_choice": {"type": "function", "function": {"name": "nope"}}},
    {"tools": [WEATHER], "tool_choice": "sometimes"},
    {"tools": [WEATHER], "tool_choice": "required", "response_format": {"type": "json_object"}},
])
def test_bad_tool_requests_are_refused(client, kw):
    assert _chat(client, **kw).status_code == 400
