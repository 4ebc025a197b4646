"""The offline `LLM` API: `chat` renders like the chat endpoint and generates the same
tokens, `embed` equals the engine's embeddings, and `generate` takes every request
feature (beam search, guided decoding) that the server does."""
import numpy as np
import pytest
from fastapi.testclient import TestClient

from rusteeze_b200.api.server import create_app
from rusteeze_b200.core.sampling_params import GuidedDecodingParams, SamplingParams
from rusteeze_b200.engine.async_engine import AsyncLLMEngine
from rusteeze_b200.engine.llm_engine import LLM


@pytest.fixture(scope="module")
def llm():
    return LLM(preset="tiny-llama", device="cpu", dtype="float32", num_gpu_blocks=96, max_num_seqs=8)


def test_chat_matches_the_chat_endpoint(llm):
    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hello there"}]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    out = llm.chat(msgs, sp)
    assert len(out) == 1
    cfg = llm.engine.config
    cfg.logging.request_logging = False
    ae = AsyncLLMEngine(llm.engine).start()
    try:
        r = TestClient(create_app(ae, cfg)).post("/v1/chat/completions", json={
            "messages": msgs, "max_tokens": 6, "temperature": 0, "ignore_eos": True})
        assert r.json()["choices"][0]["message"]["content"] == out[0].outputs[0].text
        assert r.json()["usage"]["prompt_tokens"] == len(out[0].prompt_token_ids)
    finally:
        ae.shutdown()
    two = llm.chat([msgs, [{"role": "user", "content": "x"}]], sp)
    assert len(two) == 2 and two[0].outputs[0].token_ids == out[0].outputs[0].token_ids


def test_embed_and_request_features(llm):
    v = llm.embed(["abc", [5, 6, 7]])
    assert len(v) == 2 and abs(np.linalg.norm(v[0]) - 1) < 1e-5
    assert np.allclose(v[1], llm.engine.embed([[5, 6, 7]])[0])
    assert np.allclose(v[0], llm.engine.embed([llm.tokenizer.encode("abc")])[0])
    beam = llm.generate("hi", SamplingParams(n=2, best_of=3, use_beam_search=True, temperature=0.0, max_tokens=4,
                                             ignore_eos=True))
    assert len(beam[0].outputs) == 2
    g = llm.generate(["a", "b"], SamplingParams(temperature=0.8, max_tokens=10,
                                                guided_decoding=GuidedDecodingParams(choice=["yes", "no"])))
    assert all(o.outputs[0].text in ("yes", "no") for o in g)
