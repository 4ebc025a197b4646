"""N-gram (prompt-lookup) speculative decoding: the C++ proposer against a Python restatement
of the rule (longest recurring suffix, most recent occurrence, the k tokens after it), and
the engine's output with it equal to plain greedy decoding, with proposals accepted."""
import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from rusteeze_b200 import _host
from rusteeze_b200.config.config import Config, SpeculativeSection
from rusteeze_b200.config.validation import collect_errors
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig

MC = ModelConfig(name="spec-tiny", hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2, vocab_size=512, max_position_embeddings=1024)


def lookup(t, k, n_max, n_min):
    """The rule, written plainly: for n = n_max .. n_min, the latest i with t[i:i+n] equal
    to the last n tokens and a token after it; propose t[i+n : i+n+k]."""
    L = len(t)
    for n in range(min(n_max, L - 1), n_min - 1, -1):
        pat = t[L - n:]
        for i in range(L - n - 1, -1, -1):
            if t[i:i + n] == pat:
                return t[i + n:i + n + k]
    return []


@settings(max_examples=300, deadline=None)
@given(st.lists(st.lists(st.integers(0, 5), min_size=0, max_size=60), min_size=1, max_size=6),
       st.integers(1, 6), st.integers(1, 5), st.integers(0, 3))
def test_proposer_matches_the_rule(seqs, k, n_min, extra):
    n_max = n_min + extra
    props, counts = _host.ngram_propose([np.asarray(s, dtype=np.int64) for s in seqs], k, n_max, n_min)
    assert props.shape == (len(seqs), k) and counts.shape == (len(seqs),)
    for s, row, c in zip(seqs, props, counts):
        want = lookup(s, k, n_max, n_min)
        assert int(c) == len(want)
        assert row[:c].tolist() == want
        pad = want[-1] if want else (s[-1] if s else 0)
        assert (row[c:] == pad).all()


def test_proposer_prefers_the_longest_suffix_and_the_latest_match():
    t = [1, 2, 3, 9, 2, 3, 7, 1, 2, 3]
    props, counts = _host.ngram_propose([np.asarray(t, dtype=np.int64)], 2, 3, 1)
    # "1 2 3" recurs at 0 (followed by 9 2); "2 3" alone would take the later 2 3 -> 7 1
    assert counts.tolist() == [2] and props[0].tolist() == [9, 2]
    props, counts = _host.ngram_propose([np.asarray(t, dtype=np.int64)], 2, 2, 1)
    assert props[0].tolist() == [7, 1]
    with pytest.raises(ValueError):
        _host.ngram_propose([np.asarray(t, dtype=np.int64)], 0, 2, 1)


def _engine(spec=None, num_blocks=128):
    cfg = Config()
    cfg.model.device, cfg.model.dtype = "cpu", "float32"
    cfg.engine.num_gpu_blocks = num_blocks
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 256
    cfg.engine.enable_chunked_prefill = True
    cfg.engine.speculative = spec
    return LLMEngine(cfg, model_config=MC)


def _run(eng, prompts, n=40, temps=None):
    ids = []
    for i, p in enumerate(prompts):
        t = 0.0 if temps is None else temps[i]
        ids.append(eng.add_request(None, None, SamplingParams(temperature=t, max_tokens=n, ignore_eos=True, seed=3),
                                   p).request_id)
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o.outputs[0].token_ids
    return [done[i] for i in ids]


def _prompts():
    rng = np.random.default_rng(0)
    base = rng.integers(0, 512, 30).tolist()
    # prompts that repeat themselves (the case prompt lookup is for), and one that does not
    return [base + base[:20], (base[:10] * 4), rng.integers(0, 512, 25).tolist()]


def test_ngram_greedy_equals_plain_decoding_and_accepts_proposals():
    prompts = _prompts()
    ref = _run(_engine(), prompts)
    eng = _engine(SpeculativeSection(method="ngram", num_speculative_tokens=4))
    assert eng.spec.drunner is None          # no draft model, no draft KV
    got = _run(eng, prompts)
    assert got == ref
    st_ = eng.spec.stats
    assert st_["rounds"] > 0 and st_["accepted"] > 0
    # more tokens came out than rounds + plain steps would give one at a time
    assert st_["emitted"] > st_["rounds"]


def test_ngram_mixed_with_sampled_requests_stays_exact_for_greedy_ones():
    prompts = _prompts()
    ref = _run(_engine(), prompts, temps=[0.0, 0.8, 0.0])
    got = _run(_engine(SpeculativeSection(method="ngram", num_speculative_tokens=3)), prompts,
               temps=[0.0, 0.8, 0.0])
    # the sampled request keeps the batch on plain steps while it runs; greedy outputs match
    assert got[0] == ref[0] and got[2] == ref[2]
    assert got[1] == ref[1]                  # plain steps: same seed, same sampler


def test_ngram_under_preemption_matches():
    prompts = _prompts()
    ref = _run(_engine(), prompts, n=60)
    eng = _engine(SpeculativeSection(method="ngram", num_speculative_tokens=4), num_blocks=14)
    got = _run(eng, prompts, n=60)
    assert eng.scheduler.num_preemptions > 0
    assert got == ref


def test_ngram_config_validation():
    cfg = Config()
    cfg.engine.speculative = SpeculativeSection(method="ngram", draft_preset="llama-3.2-1b")
    assert any("no draft model" in e for e in collect_errors(cfg))
    cfg.engine.speculative = SpeculativeSection(method="medusa")
    assert any("medusa" in e for e in collect_errors(cfg))
    cfg.engine.speculative = SpeculativeSection(method="ngram", ngram_min=3, ngram_max=2)
    assert any("ngram_min" in e for e in collect_errors(cfg))
    cfg.engine.speculative = SpeculativeSection(method="ngram")
    assert not collect_errors(cfg)
