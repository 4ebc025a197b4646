"""End-to-end oracle on the tiny Llama CPU fp32 configuration: the
continuously batched, paged engine must emit exactly the greedy tokens of a
naive per-request full-recompute forward (2 layers, hidden 256, 4q/2kv heads,
SwiGLU 688, vocab 32000, N(0,0.02) weights from a seed; 8 requests with
prompts uniform in [16,128]; paged KV with block 16 and 64 blocks; 32 greedy
tokens each)."""
import numpy as np
import pytest

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.naive import naive_greedy


def make_engine(num_blocks=64, max_seqs=8, max_tokens=256, chunked=True, prefix=False,
                preemption="recompute", swap_gb=0.05, preset="tiny-llama"):
    cfg = Config()
    cfg.model.preset = preset
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = num_blocks
    cfg.engine.max_num_seqs = max_seqs
    cfg.engine.max_num_batched_tokens = max_tokens
    cfg.engine.enable_chunked_prefill = chunked
    cfg.engine.enable_prefix_caching = prefix
    cfg.engine.scheduling.preemption_mode = preemption
    cfg.engine.swap_space_gb = swap_gb
    return LLMEngine(cfg)


def prompts_for(seed=0, n=8, lo=16, hi=128, vocab=32000):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, int(rng.integers(lo, hi + 1))).tolist() for _ in range(n)]


def run(eng, prompts, max_tokens=32):
    sp = SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)
    ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o
    return [done[i].outputs[0].token_ids for i in ids]


@pytest.fixture(scope="module")
def oracle():
    eng = make_engine()
    prompts = prompts_for()
    ref = [naive_greedy(eng.model, p, 32) for p in prompts]
    return prompts, ref


def test_tiny_llama_matches_naive_recompute(oracle):
    prompts, ref = oracle
    eng = make_engine()
    assert run(eng, prompts) == ref
    assert eng.bm.num_free_gpu_blocks() == 64


def test_without_chunked_prefill(oracle):
    prompts, ref = oracle
    eng = make_engine(chunked=False)
    assert run(eng, prompts) == ref


def test_without_chunked_prefill_a_prompt_longer_than_the_step_budget_still_runs(oracle):
    """Chunked prefill off, a 64-token step budget: prompts (and recompute-preempted
    sequences) longer than any step could hold are chunked anyway instead of waiting forever."""
    prompts, ref = oracle
    eng = make_engine(chunked=False, max_tokens=64, num_blocks=24)
    assert run(eng, prompts) == ref
    assert eng.scheduler.num_preemptions > 0


def test_recompute_preemption_under_memory_pressure(oracle):
    prompts, ref = oracle
    eng = make_engine(num_blocks=24)
    assert run(eng, prompts) == ref
    assert eng.scheduler.num_preemptions > 0


def test_swap_preemption_under_memory_pressure(oracle):
    prompts, ref = oracle
    eng = make_engine(num_blocks=24, preemption="swap")
    assert run(eng, prompts) == ref
    assert eng.scheduler.num_preemptions > 0
    assert eng.bm.stats()["swap_ins"] > 0


def test_prefix_cache_reuses_blocks_and_matches(oracle):
    prompts, ref = oracle
    eng = make_engine(prefix=True)
    assert run(eng, prompts[:4]) == ref[:4]
    # same prompts again: full blocks come from the prefix cache
    assert run(eng, prompts[:4]) == ref[:4]
    st = eng.bm.stats()
    assert st["prefix_block_hits"] > 0


def test_shared_prefix_different_suffixes():
    eng = make_engine(prefix=True)
    rng = np.random.default_rng(3)
    common = rng.integers(0, 32000, 48).tolist()
    ps = [common + rng.integers(0, 32000, 10).tolist() for _ in range(3)]
    ref = [naive_greedy(eng.model, p, 8) for p in ps]
    assert run(eng, ps[:1], 8) == ref[:1]
    assert run(eng, ps[1:], 8) == ref[1:]
    assert eng.bm.stats()["prefix_block_hits"] >= 6


def test_final_only_outputs_match_streamed_outputs():
    """output_kind="final_only": one output per request, at the end, with the same tokens and
    text as the per-step (delta) outputs; stop strings still end the request on time."""
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.core.sampling_params import SamplingParams
    from rusteeze_b200.engine.llm_engine import LLMEngine
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 256
    res = {}
    for kind in ("delta", "final_only"):
        eng = LLMEngine(cfg)
        counts, final = {}, {}
        for i, stop in enumerate(([], [], ["e"])):
            sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True, stop=stop, output_kind=kind)
            eng.add_request(f"r{i}", None, sp, list(range(5 + i, 40 + 3 * i)))
        while eng.has_unfinished_requests():
            for o in eng.step():
                counts[o.request_id] = counts.get(o.request_id, 0) + 1
                if o.finished:
                    final[o.request_id] = (o.outputs[0].token_ids, o.outputs[0].text, o.outputs[0].finish_reason)
        res[kind] = (counts, final)
    assert res["delta"][1] == res["final_only"][1]
    assert all(c == 1 for c in res["final_only"][0].values()) and len(res["final_only"][0]) == 3
    assert all(c > 1 for c in res["delta"][0].values())
