"""Prompt logprobs (`prompt_logprobs`, and `echo` with `logprobs` on /v1/completions): every
prompt token after the first is scored by the model at the position before it, equal to the
dense fp32 oracle, also when the prompt is longer than one step's token budget."""
import numpy as np
import pytest
import torch

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig
from rusteeze_b200.models.naive import naive_logits

MC = ModelConfig(name="tiny-plp", hidden_size=64, intermediate_size=128, num_hidden_layers=2,
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


def _run(eng, prompts, k):
    ids = [eng.add_request(None, None, SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True,
                                                      prompt_logprobs=k), p).request_id for p in prompts]
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o
    return [done[i] for i in ids]


@pytest.mark.parametrize("max_tokens", [512, 32])
def test_prompt_logprobs_match_the_oracle(max_tokens):
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 512, n).tolist() for n in (5, 70, 130)]
    eng = _engine(max_tokens)
    outs = _run(eng, prompts, 3)
    for p, o in zip(prompts, outs):
        plp = o.prompt_logprobs
        assert len(plp) == len(p) and plp[0] is None
        ref = torch.log_softmax(naive_logits(eng.model, p).double(), -1)
        for j in range(1, len(p)):
            d = plp[j]
            assert abs(d[p[j]] - float(ref[j - 1, p[j]])) < 1e-4
            top = ref[j - 1].topk(3)
            assert set(top.indices.tolist()) <= set(d)
        # the generated tokens are unaffected by the scoring pass
        assert o.outputs[0].token_ids == _plain(p)


_PLAIN = {}


def _plain(p):
    key = tuple(p)
    if key not in _PLAIN:
        eng = _engine()
        eng.add_request("x", None, SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True), p)
        out = None
        while eng.has_unfinished_requests():
            for o in eng.step():
                out = o
        _PLAIN[key] = out.outputs[0].token_ids
    return _PLAIN[key]


def test_prompt_logprobs_with_prefix_caching_and_k_zero():
    rng = np.random.default_rng(1)
    base = rng.integers(0, 512, 40).tolist()
    eng = _engine(prefix=True)
    a, b = _run(eng, [base, base + [7, 8, 9]], 0)
    assert a.prompt_logprobs[1:] == b.prompt_logprobs[1:len(base)]
    assert all(len(d) == 1 for d in b.prompt_logprobs[1:])          # k = 0: the prompt's own token only


def test_echo_logprobs_through_the_api():
    from fastapi.testclient import TestClient

    from rusteeze_b200.api.server import create_app
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    cfg = Config()
    cfg.logging.request_logging = False
    eng = _engine()
    ae = AsyncLLMEngine(eng).start()
    try:
        c = TestClient(create_app(ae, cfg))
        prompt = [11, 12, 13, 14, 15]
        r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 2, "echo": True, "logprobs": 2,
                                            "temperature": 0, "ignore_eos": True})
        assert r.status_code == 200, r.text
        lp = r.json()["choices"][0]["logprobs"]
        assert len(lp["tokens"]) == len(prompt) + 2
        assert lp["token_logprobs"][0] is None and all(x is not None for x in lp["token_logprobs"][1:])
        ref = torch.log_softmax(naive_logits(eng.model, prompt).double(), -1)
        assert abs(lp["token_logprobs"][1] - float(ref[0, prompt[1]])) < 1e-4
    finally:
        ae.shutdown()
