"""Chat streaming framing with several choices (CPU, ASGI client, byte-vocabulary model so
every token carries text): a role chunk per choice first, content deltas per choice, one
finish chunk per choice, the usage chunk (empty choices) when asked, then [DONE]; the
streamed content of each choice equals the non-streamed response with the same seed."""
import json

from fastapi.testclient import TestClient

from rusteeze_b200.api.server import create_app
from rusteeze_b200.config.config import Config
from rusteeze_b200.engine.async_engine import AsyncLLMEngine
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig

BYTES = ModelConfig(name="tiny-bytes", hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                    num_attention_heads=2, num_key_value_heads=1, vocab_size=256, max_position_embeddings=2048)


def test_chat_stream_with_two_choices_and_usage():
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 128
    cfg.logging.request_logging = False
    ae = AsyncLLMEngine(LLMEngine(cfg, model_config=BYTES)).start()
    c = TestClient(create_app(ae, cfg))
    body = {"model": "tiny-llama", "messages": [{"role": "user", "content": "hello there"}], "max_tokens": 12,
            "temperature": 0.8, "n": 2, "seed": 77, "ignore_eos": True}
    try:
        r = c.post("/v1/chat/completions", json=body)
        assert r.status_code == 200, r.text
        want = {ch["index"]: ch["message"]["content"] for ch in r.json()["choices"]}
        with c.stream("POST", "/v1/chat/completions",
                      json={**body, "stream": True, "stream_options": {"include_usage": True}}) as rs:
            lines = [ln for ln in rs.iter_lines() if ln]
    finally:
        ae.shutdown()
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
    assert all(ch["object"] == "chat.completion.chunk" for ch in chunks)
    roles = [ch["choices"][0]["index"] for ch in chunks[:2]]
    assert sorted(roles) == [0, 1] and all(ch["choices"][0]["delta"].get("role") == "assistant" for ch in chunks[:2])
    usage = chunks[-1]
    assert usage["choices"] == [] and usage["usage"]["completion_tokens"] == 24
    got, fins = {0: "", 1: ""}, {}
    for ch in chunks[2:-1]:
        (choice,) = ch["choices"]
        got[choice["index"]] += choice["delta"].get("content") or ""
        if choice.get("finish_reason"):
            assert choice["index"] not in fins
            fins[choice["index"]] = choice["finish_reason"]
    assert fins == {0: "length", 1: "length"}
    assert got == want
