"""Embeddings (`LLMEngine.embed`, /v1/embeddings): last-token and mean pooling equal the
dense fp32 oracle's final normalised hidden states, also for inputs longer than one step's
token budget; embedding never touches the prefix cache and runs between generation steps;
the API's formats (float, base64), `dimensions` and usage."""
import asyncio
import base64

import numpy as np
import pytest

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.errors import InvalidRequestError
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig
from rusteeze_b200.models.naive import naive_logits

MC = ModelConfig(name="tiny-emb", hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2, vocab_size=512, max_position_embeddings=1024)


def _engine(max_tokens=512, prefix=False):
    cfg = Config()
    cfg.model.device, cfg.model.dtype = "cpu", "float32"
    cfg.engine.num_gpu_blocks = 128
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = max_tokens
    cfg.engine.enable_chunked_prefill = True
    cfg.engine.enable_prefix_caching = prefix
    return LLMEngine(cfg, model_config=MC)


def _oracle(model, toks, pooling):
    seen = {}
    naive_logits(model, toks, observer=lambda n, x: seen.__setitem__(n, x) if n == "lm_head" else None)
    h = seen["lm_head"].double()
    v = h[-1] if pooling == "last" else h.mean(0)
    return (v / v.norm()).numpy()


@pytest.mark.parametrize("max_tokens", [512, 32])
@pytest.mark.parametrize("pooling", ["last", "mean"])
def test_embeddings_match_the_oracle(pooling, max_tokens):
    eng = _engine(max_tokens)
    rng = np.random.default_rng(0)
    inputs = [rng.integers(0, 512, n).tolist() for n in (1, 17, 100)]
    free0 = eng.bm.num_free_gpu_blocks()
    vecs = eng.embed(inputs, pooling)
    assert eng.bm.num_free_gpu_blocks() == free0             # blocks returned
    for toks, v in zip(inputs, vecs):
        assert v.shape == (MC.hidden_size,) and abs(np.linalg.norm(v) - 1) < 1e-5
        assert np.abs(v - _oracle(eng.model, toks, pooling)).max() < 1e-4
    raw = eng.embed(inputs[:1], pooling, normalize=False)[0]
    assert np.linalg.norm(raw) > 0 and abs(np.linalg.norm(raw) - 1) > 1e-3


def test_embedding_leaves_the_prefix_cache_and_running_requests_alone():
    eng = _engine(prefix=True)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 512, 64).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    eng.add_request("a", None, sp, prompt)
    eng.step()
    eng.step()
    hits0, cached0 = eng.bm.stats()["prefix_block_hits"], eng.bm.cached_prefix_len(np.asarray(prompt + [0]))
    other = rng.integers(0, 512, 48).tolist()
    v1 = eng.embed([prompt, other])[0]                         # the cached prompt's tokens, and new ones
    # no cache block was claimed by the embedding, and none of its blocks was published
    assert eng.bm.stats()["prefix_block_hits"] == hits0
    assert eng.bm.cached_prefix_len(np.asarray(prompt + [0])) == cached0
    assert eng.bm.cached_prefix_len(np.asarray(other + [0])) == 0
    out = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            out = o
    ref = _engine()
    ref.add_request("a", None, sp, prompt)
    ref_out = None
    while ref.has_unfinished_requests():
        for o in ref.step():
            ref_out = o
    assert out.outputs[0].token_ids == ref_out.outputs[0].token_ids
    assert np.abs(v1 - _oracle(eng.model, prompt, "last")).max() < 1e-4


def test_bad_inputs_are_refused():
    eng = _engine()
    for inputs, exc in (([[]], InvalidRequestError), ([[600]], InvalidRequestError)):
        with pytest.raises(exc):
            eng.embed(inputs)
    with pytest.raises(InvalidRequestError):
        eng.embed([[1, 2]], pooling="max")


def test_embeddings_api():
    from fastapi.testclient import TestClient

    from rusteeze_b200.api.server import create_app
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    cfg = Config()
    cfg.logging.request_logging = False
    eng = _engine()
    ae = AsyncLLMEngine(eng).start()
    try:
        c = TestClient(create_app(ae, cfg))
        r = c.post("/v1/embeddings", json={"input": [[5, 6, 7], [8, 9]]})
        assert r.status_code == 200, r.text
        d = r.json()
        assert d["object"] == "list" and [x["index"] for x in d["data"]] == [0, 1]
        assert d["usage"] == {"prompt_tokens": 5, "total_tokens": 5}
        v0 = np.array(d["data"][0]["embedding"])
        assert np.abs(v0 - _oracle(eng.model, [5, 6, 7], "last")).max() < 1e-4
        r = c.post("/v1/embeddings", json={"input": [5, 6, 7], "encoding_format": "base64", "dimensions": 16})
        b = np.frombuffer(base64.b64decode(r.json()["data"][0]["embedding"]), dtype="<f4")
        want = v0[:16] / np.linalg.norm(v0[:16])
        assert b.shape == (16,) and np.abs(b - want).max() < 1e-5
        r = c.post("/v1/embeddings", json={"input": "hello there", "pooling": "mean"})
        assert r.status_code == 200 and len(r.json()["data"][0]["embedding"]) == MC.hidden_size
        assert c.post("/v1/embeddings", json={"input": []}).status_code == 400
        assert c.post("/v1/embeddings", json={"input": [1, 2], "dimensions": 1000}).status_code == 400
    finally:
        ae.shutdown()


def test_embedding_while_generation_streams():
    """An embedding job submitted while requests are decoding runs between their steps."""
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    eng = _engine()
    ae = AsyncLLMEngine(eng).start()

    async def main():
        async def gen():
            last = None
            async for o in ae.generate(None, SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True), "g",
                                       list(range(10, 40))):
                last = o
            return last

        t = asyncio.ensure_future(gen())
        await asyncio.sleep(0.05)
        vecs = await ae.embed([[1, 2, 3]])
        return vecs, await t

    try:
        vecs, last = asyncio.run(main())
    finally:
        ae.shutdown()
    assert last.finished and len(last.outputs[0].token_ids) == 30
    assert np.abs(vecs[0] - _oracle(eng.model, [1, 2, 3], "last")).max() < 1e-4
