"""Request-surface fuzzing (CPU): random sampling parameters, including edge values
(NaN and infinite floats, token ids outside the vocabulary, huge n / best_of / logprobs,
tiny caches), are either refused when the request is added or served to the end.
No request may raise inside `step()`, because a failing step takes the whole engine
(and every other client's request) down."""
import math
import random

import pytest

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.errors import RusteezeError
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine

_EDGE_FLOATS = [0.0, -0.0, 1e-9, 0.5, 1.0, 2.0, -1.0, 1e9, float("nan"), float("inf"), -float("inf")]


def _engine(blocks=24, max_seqs=4):
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.model.max_model_len = 128
    cfg.engine.num_gpu_blocks = blocks
    cfg.engine.max_num_seqs = max_seqs
    cfg.engine.max_num_batched_tokens = 128
    cfg.engine.enable_chunked_prefill = True
    return LLMEngine(cfg)


def _random_params(rng, V):
    def f():
        return rng.choice(_EDGE_FLOATS) if rng.random() < 0.3 else rng.uniform(0, 1.5)

    def tok():
        return rng.choice([0, 1, V - 1, V, V + 7, -1, 10 ** 9]) if rng.random() < 0.4 else rng.randrange(V)
    kw = {}
    keys = ["temperature", "top_p", "min_p", "typical_p", "frequency_penalty", "presence_penalty",
            "repetition_penalty", "eta_cutoff", "epsilon_cutoff", "mirostat_tau", "mirostat_eta"]
    for k in rng.sample(keys, rng.randint(0, 5)):
        kw[k] = f()
    if rng.random() < 0.3:
        kw["top_k"] = rng.choice([-1, 0, 1, 2, 5, V, V + 100, -5])
    if rng.random() < 0.3:
        kw["n"] = rng.choice([1, 2, 3, 9])
        kw["best_of"] = kw["n"] + rng.choice([0, 0, 1, 5])
    if rng.random() < 0.3:
        kw["logit_bias"] = {tok(): rng.choice([-100.0, 5.0, 100.0, float("nan"), 1e9]) for _ in range(3)}
    if rng.random() < 0.3:
        kw["stop_token_ids"] = [tok() for _ in range(2)]
        kw["min_tokens"] = rng.choice([0, 2, 5])
    if rng.random() < 0.2:
        kw["mirostat_mode"] = rng.choice([0, 1, 2, 3])
    if rng.random() < 0.3:
        kw["logprobs"] = rng.choice([0, 1, 5, V + 10, -1])
    if rng.random() < 0.2:
        kw["seed"] = rng.choice([0, -1, 2 ** 64 + 3, -2 ** 70])
    kw["max_tokens"] = rng.choice([1, 4, 9, 300]) if rng.random() < 0.9 else rng.choice([0, -3])
    kw["ignore_eos"] = rng.random() < 0.5
    return kw


@pytest.mark.parametrize("seed", range(4))
def test_random_requests_are_refused_or_served(seed):
    rng = random.Random(seed)
    eng = _engine(blocks=rng.choice([12, 24, 64]), max_seqs=rng.choice([2, 4, 8]))
    V = eng.model_config.vocab_size
    added, refused = [], 0
    for i in range(40):
        kw = _random_params(rng, V)
        prompt = [rng.randrange(V) for _ in range(rng.randint(1, 40))]
        if rng.random() < 0.1:
            prompt[rng.randrange(len(prompt))] = rng.choice([V, -1])
        try:
            eng.add_request(f"r{i}", None, SamplingParams(**kw), prompt_token_ids=prompt)
            added.append(f"r{i}")
        except RusteezeError:
            refused += 1
        for _ in range(rng.randint(0, 2)):
            if eng.has_unfinished_requests():
                eng.step()
    finished = set()
    for _ in range(5000):
        if not eng.has_unfinished_requests():
            break
        for o in eng.step():
            if o.finished:
                finished.add(o.request_id)
                for c in o.outputs:
                    assert all(0 <= t < V for t in c.token_ids)
                    assert all(not math.isnan(v) for v in (c.cumulative_logprob,) if v is not None)
    assert not eng.has_unfinished_requests()
    assert refused > 0 and added
    # the engine still serves a plain request afterwards
    eng.add_request("after", None, SamplingParams(max_tokens=3, ignore_eos=True, temperature=0),
                    prompt_token_ids=[1, 2, 3])
    outs = []
    while eng.has_unfinished_requests():
        outs += eng.step()
    assert outs[-1].finished and len(outs[-1].outputs[0].token_ids) == 3


@pytest.mark.parametrize("field,value", [
    ("temperature", float("nan")), ("temperature", float("inf")), ("repetition_penalty", float("nan")),
    ("mirostat_tau", float("nan")), ("eta_cutoff", float("inf")), ("epsilon_cutoff", -0.5),
])
def test_non_finite_or_out_of_range_floats_are_refused(field, value):
    with pytest.raises(RusteezeError):
        SamplingParams(**{field: value})


@pytest.mark.parametrize("kw", [
    {"logit_bias": {10 ** 6: 1.0}}, {"logit_bias": {-1: 1.0}},
    {"stop_token_ids": [10 ** 6], "min_tokens": 2}, {"stop_token_ids": [-3]},
])
def test_token_ids_outside_the_vocabulary_are_refused_at_admission(kw):
    eng = _engine()
    with pytest.raises(RusteezeError):
        eng.add_request("x", None, SamplingParams(max_tokens=2, **kw), prompt_token_ids=[1, 2])
    assert not eng.has_unfinished_requests()
