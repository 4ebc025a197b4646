"""HTTP request fuzzing on the tiny CPU model: random JSON bodies for the completion
and chat endpoints -- wrong types, missing fields, edge numbers, token ids outside
the vocabulary, odd chat content -- get a 2xx or a 4xx with an OpenAI error body,
never a 500, and the engine stays ready and serves a plain request afterwards."""
import json
import random

import pytest
from fastapi.testclient import TestClient

from rusteeze_b200.api.server import create_app
from rusteeze_b200.config.config import Config
from rusteeze_b200.engine.async_engine import AsyncLLMEngine
from rusteeze_b200.engine.llm_engine import LLMEngine

_VALUES = [None, True, 0, 1, -1, 3, 2 ** 31, 2 ** 63, -2 ** 63, 0.5, -0.5, 1e308, "x", "", [], {}, [1, 2],
           ["a"], {"a": 1}]
_NUM_FIELDS = ["max_tokens", "temperature", "top_p", "top_k", "min_p", "n", "best_of", "presence_penalty",
               "frequency_penalty", "repetition_penalty", "seed", "priority", "min_tokens", "logprobs",
               "top_logprobs", "max_completion_tokens"]


def _cfg():
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.model.max_model_len = 96
    cfg.engine.num_gpu_blocks = 48
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 128
    cfg.server.timeout_seconds = 30
    cfg.logging.request_logging = False
    return cfg


def _body(rng, chat, V):
    b = {}
    if chat:
        msgs = rng.choice([
            [{"role": "user", "content": "hi"}],
            [{"role": "system", "content": "s"}, {"role": "user", "content": [{"type": "text", "text": "a"}]}],
            [{"role": "user"}], [], [{"content": "no role"}], "hello", [{"role": "tool", "content": None}],
            [{"role": "user", "content": [{"type": "image_url", "image_url": {"url": "x"}}]}],
        ])
        if rng.random() < 0.95:
            b["messages"] = msgs
    else:
        p = rng.choice(["abc", "", ["a", "b"], [1, 2, 3], [[1, 2], [3]], [V, 1], [-1], [[]], [], 5, None,
                        "word " * 200])
        if rng.random() < 0.95:
            b["prompt"] = p
    for k in rng.sample(_NUM_FIELDS, rng.randint(0, 6)):
        b[k] = rng.choice(_VALUES) if rng.random() < 0.5 else rng.choice([0, 1, 2, 4])
    if rng.random() < 0.2:
        b["logit_bias"] = rng.choice([{"5": 1.0}, {str(V + 1): 1.0}, {"-2": 3.0}, {"x": 1.0}, {"5": 1e6}, []])
    if rng.random() < 0.2:
        b["stop_token_ids"] = rng.choice([[1], [V], [-1], ["a"], None])
    if rng.random() < 0.2:
        b["stop"] = rng.choice(["\n", ["a", "b"], "", [""], 5, ["x"] * 10])
    if rng.random() < 0.3:
        b["stream"] = rng.choice([True, False, "yes"])
    if rng.random() < 0.1:
        b["stream_options"] = rng.choice([{"include_usage": True}, {"include_usage": "no"}, 1])
    if rng.random() < 0.1:
        b["model"] = rng.choice(["tiny-llama", "other", 7])
    if rng.random() < 0.1:
        b["response_format"] = rng.choice([
            {"type": "json_object"}, {"type": "nope"}, "x", {"type": "json_schema"},
            {"type": "json_schema", "json_schema": {"schema": {"type": "integer"}}},
            {"type": "json_schema", "json_schema": {"schema": 5}}, {"type": "json_schema", "json_schema": []}])
    if rng.random() < 0.1:
        b["guided_regex"] = rng.choice(["[a-z]{2}", "(", "a{99999}", "(?=x)", 5, None, ""])
    if rng.random() < 0.1:
        b["guided_choice"] = rng.choice([["a", "b"], [], "x", [1], [""]])
    if rng.random() < 0.1:
        b["guided_json"] = rng.choice([{"type": "object"}, {"type": "weird"}, "not json", '{"type": "boolean"}',
                                       {"$ref": "#/nowhere"}, {"enum": []}, 3])
    if rng.random() < 0.1:
        b["use_beam_search"] = rng.choice([True, False, "x"])
        b["length_penalty"] = rng.choice([1.0, -2.0, 0, "x", 1e308])
        b["early_stopping"] = rng.choice([True, False, "never", "sometimes", 3])
    if chat and rng.random() < 0.15:
        b["tools"] = rng.choice([
            [{"type": "function", "function": {"name": "f", "parameters": {"type": "object",
                                                                          "properties": {"a": {"type": "integer"}}}}}],
            [{"type": "function"}], "x", [5], [], [{"type": "function", "function": {"name": "f", "parameters": 7}}]])
        b["tool_choice"] = rng.choice(["auto", "none", "required", {"type": "function", "function": {"name": "f"}},
                                       {"type": "x"}, 7, None])
    if not chat and rng.random() < 0.1:
        b["echo"] = rng.choice([True, False])
    b.setdefault("max_tokens", rng.choice([1, 3, 5]))
    return b


@pytest.fixture(scope="module")
def client():
    cfg = _cfg()
    ae = AsyncLLMEngine(LLMEngine(cfg)).start()
    c = TestClient(create_app(ae, cfg), raise_server_exceptions=False)
    yield c, ae
    ae.shutdown()


def _post(c, url, body):
    if body.get("stream") is True:
        with c.stream("POST", url, json=body) as r:
            return r.status_code, "".join(r.iter_text())
    r = c.post(url, json=body)
    return r.status_code, r.text


@pytest.mark.parametrize("seed", range(3))
def test_random_bodies_never_get_a_server_error(client, seed):
    c, ae = client
    V = ae.engine.model_config.vocab_size
    rng = random.Random(seed)
    codes = {}
    for _ in range(60):
        chat = rng.random() < 0.5
        body = _body(rng, chat, V)
        url = "/v1/chat/completions" if chat else "/v1/completions"
        code, text = _post(c, url, body)
        codes[code] = codes.get(code, 0) + 1
        assert code < 500, (body, code, text[:400])
        if code == 200 and body.get("stream") is True:
            assert text.rstrip().endswith("data: [DONE]"), (body, text[-300:])
        if code >= 400:
            err = json.loads(text)
            assert "error" in err or "detail" in err, text[:300]
        assert ae.is_ready, (body, ae.last_error)
    assert codes.get(200, 0) > 0 and sum(v for k, v in codes.items() if k >= 400) > 0, codes
    code, text = _post(c, "/v1/completions", {"prompt": "fine", "max_tokens": 2, "ignore_eos": True})
    assert code == 200 and json.loads(text)["usage"]["completion_tokens"] == 2


@pytest.mark.parametrize("body", [
    {"prompt": [1, 2, 3], "top_k": 2 ** 63, "temperature": 0.5},                 # overflowed the sampler
    {"prompt": [1, 2, 3], "use_beam_search": True, "best_of": 2, "length_penalty": 1e308},
    {"prompt": [1, 2, 3], "guided_json": {"enum": []}},                          # crashed the NFA builder
    {"prompt": [1, 2, 3], "guided_regex": ""},
])
def test_inputs_that_once_broke_the_engine_are_refused_or_served(client, body):
    c, ae = client
    code, text = _post(c, "/v1/completions", dict(body, max_tokens=3))
    assert code < 500, text[:300]
    assert ae.is_ready, ae.last_error
    code, _ = _post(c, "/v1/completions", {"prompt": "fine", "max_tokens": 2})
    assert code == 200


@pytest.mark.parametrize("seed", range(2))
def test_random_embedding_and_tokenizer_bodies_never_get_a_server_error(client, seed):
    c, ae = client
    V = ae.engine.model_config.vocab_size
    rng = random.Random(100 + seed)
    for _ in range(40):
        url = rng.choice(["/v1/embeddings", "/tokenize", "/detokenize"])
        body = {}
        if url == "/v1/embeddings":
            if rng.random() < 0.9:
                body["input"] = rng.choice(["abc", "", ["a", "bb"], [1, 2, 3], [[1], [2, 3]], [[]], [V], [-1], 5,
                                            None, "w " * 300, [[1] * 200]])
            for k, vals in (("encoding_format", ["float", "base64", "hex", 1]), ("dimensions", [1, 8, 0, -1, 10 ** 6, "x"]),
                            ("pooling", ["last", "mean", "max"]), ("normalize", [True, False, "x"])):
                if rng.random() < 0.3:
                    body[k] = rng.choice(vals)
        elif url == "/tokenize":
            for k, vals in (("prompt", ["hi", "", 5, None]), ("messages", [[{"role": "user", "content": "x"}], [], "x"]),
                            ("add_special_tokens", [True, False, "x"])):
                if rng.random() < 0.5:
                    body[k] = rng.choice(vals)
        else:
            body["tokens"] = rng.choice([[5, 6], [], [V], [-1], "x", [1.5], None])
        code, text = _post(c, url, body)
        assert code < 500, (url, body, code, text[:400])
        assert ae.is_ready
    assert c.post("/v1/embeddings", json={"input": "fine"}).status_code == 200


def test_request_chat_templates_need_the_operator_s_consent():
    """A chat request's own Jinja template is refused unless the server trusts request
    templates; a trusted template that fails to render is the client's error (400)."""
    body = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 2, "ignore_eos": True,
            "chat_template": "{% for i in range(99999) %}{% for j in range(99999) %}x{% endfor %}{% endfor %}"}
    for trusted in (False, True):
        cfg = _cfg()
        cfg.server.trust_request_chat_template = trusted
        ae = AsyncLLMEngine(LLMEngine(cfg)).start()
        c = TestClient(create_app(ae, cfg), raise_server_exceptions=False)
        try:
            if not trusted:
                r = c.post("/v1/chat/completions", json=body)
                assert r.status_code == 400 and "chat_template" in r.text
                continue
            ok = {**body, "chat_template": "{% for m in messages %}<{{ m.role }}>{{ m.content }}{% endfor %}"}
            assert c.post("/v1/chat/completions", json=ok).status_code == 200
            for bad in ("{% if %}", "{{ raise_exception('roles must alternate') }}", "{{ messages[5].content }}x"):
                r = c.post("/v1/chat/completions", json={**body, "chat_template": bad})
                assert r.status_code == 400, (bad, r.status_code, r.text)
        finally:
            ae.shutdown()


def test_request_bodies_above_the_limit_get_413():
    cfg = _cfg()
    cfg.server.max_body_bytes = 4096
    ae = AsyncLLMEngine(LLMEngine(cfg)).start()
    c = TestClient(create_app(ae, cfg), raise_server_exceptions=False)
    try:
        ok = {"prompt": "small", "max_tokens": 1}
        assert c.post("/v1/completions", json=ok).status_code == 200
        big = {"prompt": "x" * 10000, "max_tokens": 1}
        r = c.post("/v1/completions", json=big)                    # Content-Length over the limit
        assert r.status_code == 413 and r.json()["error"]["code"] == "payload_too_large"
        data = json.dumps(big).encode()

        def chunks():                                              # no Content-Length: counted
            for i in range(0, len(data), 1000):
                yield data[i:i + 1000]
        r = c.post("/v1/completions", content=chunks(), headers={"content-type": "application/json"})
        assert r.status_code == 413
        small = json.dumps(ok).encode()
        r = c.post("/v1/completions", content=iter([small[:5], small[5:]]),
                   headers={"content-type": "application/json"})
        assert r.status_code == 200
        assert ae.is_ready
    finally:
        ae.shutdown()
