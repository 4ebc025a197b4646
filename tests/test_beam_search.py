"""Beam search through the paged engine (CPU, fp32) against a brute-force beam search over the
dense oracle model: same hypotheses, scores and finish reasons for several widths, length
penalties, early-stopping modes and EOS pressure; width 1 equals greedy decoding; the
search survives preemption; outputs through the HTTP API."""
import json
import math

import numpy as np
import pytest
import torch

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.errors import InvalidRequestError
from rusteeze_b200.core.sampling_params import EarlyStoppingMode, SamplingParams
from rusteeze_b200.engine.beam_search import beam_score
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig
from rusteeze_b200.models.naive import naive_greedy, naive_logits

# a small vocabulary keeps the logprob gaps between candidates wide (no near-ties)
MC = ModelConfig(name="tiny-beam", hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2, vocab_size=512, max_position_embeddings=2048)


def _engine(num_blocks=128, max_seqs=16, max_tokens=512, preemption="recompute"):
    cfg = Config()
    cfg.model.device, cfg.model.dtype = "cpu", "float32"
    cfg.engine.num_gpu_blocks = num_blocks
    cfg.engine.max_num_seqs = max_seqs
    cfg.engine.max_num_batched_tokens = max_tokens
    cfg.engine.enable_chunked_prefill = True
    cfg.engine.scheduling.preemption_mode = preemption
    return LLMEngine(cfg, model_config=MC)


@torch.no_grad()
def oracle_beam(model, prompt, W, max_tokens, eos, lp_pen=1.0, early="false", bias=None, n=1):
    """Textbook beam search on the dense model: 2W candidates per step over all beams,
    EOS candidates among the first W become hypotheses, the best W others continue."""
    live = [(0.0, [])]
    fin = []

    def score(cum, L):
        return cum / (max(1, L) ** lp_pen)

    def keep(cum, toks, reason):
        fin.append((score(cum, len(toks)), cum, toks, reason))
        fin.sort(key=lambda t: -t[0])
        del fin[W:]

    for _ in range(max_tokens):
        cands = []
        for b, (cum, out) in enumerate(live):
            x = naive_logits(model, list(prompt) + out)[-1].double()
            if bias:
                for t, v in bias.items():
                    x[t] += v
            lsm = torch.log_softmax(x, -1)
            v, ix = lsm.topk(2 * W)
            cands += [(cum + float(l), b, int(t), float(l)) for l, t in zip(v, ix)]
        cands.sort(key=lambda c: -c[0])
        nxt = []
        for rank, (sc, b, t, l) in enumerate(cands[:2 * W]):
            if t in eos:
                if rank < W:
                    keep(sc, live[b][1] + [t], "stop")
                continue
            nxt.append((sc, live[b][1] + [t]))
            if len(nxt) == W:
                break
        live = nxt
        if live and len(live[0][1]) >= max_tokens:
            for cum, toks in live:
                keep(cum, toks, "length")
            live = []
        if not live:
            break
        if len(fin) >= W:
            best = max(c for c, _ in live)
            if early == "true":
                break
            L = max_tokens if (early == "never" and lp_pen > 0) else len(live[0][1])
            if fin[-1][0] >= score(best, L):
                break
    return fin[:n]


def _run(eng, prompt, params):
    eng.add_request("r", None, params, prompt)
    outs = []
    while eng.has_unfinished_requests():
        outs += eng.step()
    fin = [o for o in outs if o.finished]
    assert len(fin) == 1
    return fin[0]


def _prompt(seed, n=12):
    return np.random.default_rng(seed).integers(1, MC.vocab_size, n).tolist()


@pytest.mark.parametrize("W,n,lp,early,eos_bias", [
    (1, 1, 1.0, "false", 0.0), (2, 2, 1.0, "false", 0.0), (4, 2, 1.0, "false", 0.2),
    (4, 4, 0.5, "true", 0.4), (3, 1, 2.0, "never", 0.3), (8, 3, 1.0, "false", 0.4), (8, 8, 0.0, "never", 0.2)])
def test_beam_search_matches_the_oracle(W, n, lp, early, eos_bias):
    eng = _engine()
    eos = tuple(eng.eos_ids)
    bias = {eos[0]: eos_bias} if eos_bias else {}
    prompt = _prompt(W * 7 + n)
    params = SamplingParams(n=n, best_of=W, use_beam_search=True, temperature=0.0, max_tokens=10,
                            length_penalty=lp, early_stopping=EarlyStoppingMode(early), logit_bias=bias,
                            logprobs=0)
    out = _run(eng, prompt, params)
    want = oracle_beam(eng.model, prompt, W, 10, set(eos), lp, early, bias, n)
    assert [o.index for o in out.outputs] == list(range(len(want)))
    assert [o.token_ids for o in out.outputs] == [w[2] for w in want]
    assert [o.finish_reason for o in out.outputs] == [w[3] for w in want]
    for o, w in zip(out.outputs, want):
        assert math.isclose(o.cumulative_logprob, w[1], abs_tol=1e-3)
        assert math.isclose(beam_score(o.cumulative_logprob, len(o.token_ids), lp), w[0], abs_tol=1e-3)
    # every beam's KV blocks are back in the pool
    assert eng.bm.num_free_gpu_blocks() == eng.bm.num_gpu_blocks
    assert not eng.requests


def test_eos_pressure_yields_stop_and_length_hypotheses():
    """With a small EOS bias some hypotheses end in EOS and others at max_tokens; both are
    ranked together by the length-normalised score."""
    eng = _engine()
    eos = tuple(eng.eos_ids)
    prompt = _prompt(6)
    params = SamplingParams(n=4, best_of=4, use_beam_search=True, temperature=0.0, max_tokens=8,
                            logit_bias={eos[0]: 0.4})
    out = _run(eng, prompt, params)
    want = oracle_beam(eng.model, prompt, 4, 8, set(eos), 1.0, "false", {eos[0]: 0.4}, 4)
    assert [o.token_ids for o in out.outputs] == [w[2] for w in want]
    assert {o.finish_reason for o in out.outputs} == {"stop", "length"}
    stops = [o for o in out.outputs if o.finish_reason == "stop"]
    assert all(o.token_ids[-1] == eos[0] for o in stops)


def test_width_one_is_greedy():
    eng = _engine()
    prompt = _prompt(9)
    out = _run(eng, prompt, SamplingParams(best_of=1, use_beam_search=True, temperature=0.0, max_tokens=12,
                                           ignore_eos=True))
    assert out.outputs[0].token_ids == naive_greedy(eng.model, prompt, 12)


def test_beams_share_the_prompt_blocks_and_fork_copy_on_write():
    """The prompt's KV is computed once: a long prompt with 4 beams holds about one copy
    of its blocks, not four."""
    eng = _engine(num_blocks=256)
    prompt = _prompt(3, 200)
    eng.add_request("r", None, SamplingParams(best_of=4, use_beam_search=True, temperature=0.0, max_tokens=6,
                                              ignore_eos=True), prompt)
    eng.step()                    # prefill (chunked in one step) and the first beam step
    eng.step()
    used = eng.bm.num_gpu_blocks - eng.bm.num_free_gpu_blocks()
    assert used < 200 // 16 + 1 + 4 * 2
    while eng.has_unfinished_requests():
        eng.step()


@pytest.mark.parametrize("preemption", ["recompute", "swap"])
def test_beam_search_under_preemption_matches_the_unpressured_run(preemption):
    """A cache too small for everything at once preempts beams; the search waits for the
    preempted ones and ends with the same hypotheses."""
    prompts = [_prompt(20 + i, 40) for i in range(3)]
    params = SamplingParams(n=2, best_of=3, use_beam_search=True, temperature=0.0, max_tokens=24, ignore_eos=True)

    def run(eng):
        for i, p in enumerate(prompts):
            eng.add_request(f"r{i}", None, params, p)
        got = {}
        while eng.has_unfinished_requests():
            for o in eng.step():
                if o.finished:
                    got[o.request_id] = [c.token_ids for c in o.outputs]
        return got

    free = run(_engine(num_blocks=256))
    tight_eng = _engine(num_blocks=20, preemption=preemption)
    tight = run(tight_eng)
    assert tight_eng.scheduler.num_preemptions > 0
    assert tight == free


def test_beam_search_is_rejected_where_it_cannot_run():
    eng = _engine(max_seqs=4)
    with pytest.raises(InvalidRequestError):
        eng.add_request("r", None, SamplingParams(best_of=8, use_beam_search=True, temperature=0.0), [1, 2, 3])
    with pytest.raises(InvalidRequestError):
        SamplingParams(best_of=2, use_beam_search=True, temperature=0.7)


def test_abort_mid_search_frees_every_beam():
    eng = _engine()
    eng.add_request("r", None, SamplingParams(best_of=4, use_beam_search=True, temperature=0.0, max_tokens=50,
                                              ignore_eos=True), _prompt(4))
    for _ in range(4):
        eng.step()
    assert eng.abort_request("r")
    assert eng.bm.num_free_gpu_blocks() == eng.bm.num_gpu_blocks
    assert not eng.has_unfinished_requests()


def test_beam_search_through_the_http_api():
    """`use_beam_search` on /v1/completions: n choices ranked best first, equal to the
    oracle's search; a streamed beam request sends its text once, at the end."""
    from fastapi.testclient import TestClient

    from rusteeze_b200.api.server import create_app
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    eng = _engine()
    prompt = _prompt(11)
    want = oracle_beam(eng.model, prompt, 4, 6, set(eng.eos_ids), 1.0, "false", None, 2)
    cfg = Config()
    cfg.logging.request_logging = False
    ae = AsyncLLMEngine(eng).start()
    try:
        c = TestClient(create_app(ae, cfg))
        body = {"prompt": prompt, "max_tokens": 6, "n": 2, "best_of": 4, "use_beam_search": True,
                "logprobs": 0}
        r = c.post("/v1/completions", json=body)
        assert r.status_code == 200, r.text
        ch = r.json()["choices"]
        assert [x["index"] for x in ch] == [0, 1]
        assert [x["text"] for x in ch] == [eng.tokenizer.decode(w[2], True) for w in want]
        assert [len(x["logprobs"]["tokens"]) for x in ch] == [len(w[2]) for w in want]
        assert [x["finish_reason"] for x in ch] == [w[3] for w in want]
        r = c.post("/v1/completions", json=dict(body, stream=True))
        chunks = [json.loads(ln[6:]) for ln in r.text.splitlines() if ln.startswith("data: {")]
        texts = {}
        for k in chunks:
            for x in k["choices"]:
                texts.setdefault(x["index"], []).append(x["text"])
        assert all(sum(1 for t in texts[i] if t) <= 1 for i in (0, 1))
        assert ["".join(texts[i]) for i in (0, 1)] == [x["text"] for x in ch]
        r = c.post("/v1/completions", json=dict(body, temperature=0.7))
        assert r.status_code == 400
    finally:
        ae.shutdown()
