"""Tensor parallelism on CPU gloo ranks (worlds 2, 4 and 8): the rank-0 engine with its
worker processes must produce the same greedy tokens as the single-process engine; plan
broadcast goes over the shared-memory ring."""
import numpy as np
import pytest

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig


def _cfg(tp):
    cfg = Config()
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.model.tensor_parallel_size = tp
    cfg.engine.num_gpu_blocks = 96
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 128
    cfg.engine.enable_chunked_prefill = True
    cfg.engine.comm_backend = "nccl"
    return cfg


MC = ModelConfig(name="tp-tiny", hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2, vocab_size=1000, rms_norm_eps=1e-5,
                 max_position_embeddings=512)


def _run(eng, prompts, n=6):
    sp = SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True)
    ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o.outputs[0].token_ids
    return [done[i] for i in ids]


@pytest.mark.timeout(300)
def test_tp2_gloo_matches_single_process():
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (30, 77, 5)]
    ref = _run(LLMEngine(_cfg(1), model_config=MC), prompts)
    launcher = TPEngineLauncher(_cfg(2), model_config=MC, device_type="cpu")
    try:
        got = _run(launcher.engine(), prompts)
    finally:
        launcher.shutdown()
    assert got == ref


@pytest.mark.timeout(300)
def test_tp2_gloo_mixtral_expert_parallel_matches_single_process():
    """Mixtral-style MoE at TP2: attention heads split, experts split over the
    ranks (EP2), partial expert outputs summed -- tokens equal the 1-process run."""
    from rusteeze_b200.models.config import ModelArchitecture
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    mc = ModelConfig(name="ep-tiny", architecture=ModelArchitecture.MIXTRAL, hidden_size=128,
                     intermediate_size=192, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                     vocab_size=1000, rms_norm_eps=1e-5, max_position_embeddings=512, num_local_experts=4,
                     num_experts_per_tok=2)
    assert mc.is_moe
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (40, 9)]
    ref = _run(LLMEngine(_cfg(1), model_config=mc), prompts)
    launcher = TPEngineLauncher(_cfg(2), model_config=mc, device_type="cpu")
    try:
        got = _run(launcher.engine(), prompts)
    finally:
        launcher.shutdown()
    assert got == ref


@pytest.mark.timeout(300)
def test_dead_worker_is_reported_not_hung():
    """Failure injection on the host: the worker process of a gloo TP2 engine is
    killed between steps; rank 0's next step raises DistributedError at once
    (liveness check before the plan is published) instead of blocking in a
    collective, and shutdown completes."""
    import os
    import time
    from rusteeze_b200.core.errors import DistributedError
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    os.environ["RZ_PG_TIMEOUT_S"] = "20"
    rng = np.random.default_rng(2)
    launcher = TPEngineLauncher(_cfg(2), model_config=MC, device_type="cpu")
    try:
        eng = launcher.engine()
        sp = SamplingParams(temperature=0.0, max_tokens=50, ignore_eos=True)
        eng.add_request(None, None, sp, rng.integers(0, 1000, 20).tolist())
        for _ in range(3):
            eng.step()
        victim = launcher.procs[0]
        victim.kill()                       # our own child process, by handle
        victim.join(10)
        assert launcher.dead_workers() == [1]
        t0 = time.monotonic()
        with pytest.raises(DistributedError):
            eng.step()
        assert time.monotonic() - t0 < 5.0
    finally:
        os.environ.pop("RZ_PG_TIMEOUT_S", None)
        t1 = time.monotonic()
        launcher.shutdown(timeout=5.0)
        assert time.monotonic() - t1 < 60.0


@pytest.mark.timeout(300)
def test_tp2_timer_is_max_over_ranks():
    """TPExecutor.timer: the workers mark the window when they consume the control
    message and join one MAX all-reduce on stop; steps inside the window still run."""
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, 1000, 20).tolist() for _ in range(2)]
    launcher = TPEngineLauncher(_cfg(2), model_config=MC, device_type="cpu")
    try:
        eng = launcher.engine()
        eng.runner.timer("start")
        got = _run(eng, prompts, n=4)
        ms = eng.runner.timer("stop")
        again = _run(eng, prompts, n=4)       # the plan stream continues after the window
    finally:
        launcher.shutdown()
    assert ms is not None and ms > 0.0
    assert got == again and all(len(t) == 4 for t in got)


@pytest.mark.timeout(300)
@pytest.mark.parametrize("draft", ["self", "separate"])
def test_tp2_speculative_decoding_matches_single_process(draft, tmp_path):
    """Speculative decoding on a tensor-parallel engine: the verify (and self-draft)
    forwards go through the plan ring so every rank runs them; a separate draft model
    stays unsharded on rank 0.  Greedy output equals the non-speculative engine's."""
    import dataclasses
    from rusteeze_b200.config.config import SpeculativeSection
    from rusteeze_b200.models.loader import build_model, save_hf_checkpoint
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (12, 33)]
    ref = _run(LLMEngine(_cfg(1), model_config=MC), prompts, n=7)
    if draft == "self":
        spec = SpeculativeSection(num_speculative_tokens=3)
    else:
        dmc = dataclasses.replace(MC, name="tp-tiny-draft", num_hidden_layers=1)
        save_hf_checkpoint(build_model(dmc, dtype=__import__("torch").float32, seed=5), str(tmp_path))
        spec = SpeculativeSection(draft_model=str(tmp_path), num_speculative_tokens=3)
    cfg = _cfg(2)
    cfg.engine.speculative = spec
    launcher = TPEngineLauncher(cfg, model_config=MC, device_type="cpu")
    try:
        eng = launcher.engine()
        got = _run(eng, prompts, n=7)
        stats = dict(eng.spec.stats)
    finally:
        launcher.shutdown()
    assert got == ref
    assert stats["rounds"] > 0
    if draft == "self":
        assert stats["accepted"] == stats["proposed"]


@pytest.mark.timeout(300)
def test_tp2_fp8_quantises_each_shard_like_the_full_model():
    """Block-scaled FP8 at TP2: every rank quantises its own shard; with shard
    boundaries on 128-element blocks that equals quantising the full model, so the
    greedy tokens match the single-process FP8 engine."""
    from rusteeze_b200.config.config import QuantizationConfig
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    mc = ModelConfig(name="tp-fp8", hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                     num_attention_heads=8, num_key_value_heads=4, vocab_size=1024, rms_norm_eps=1e-5,
                     max_position_embeddings=512)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 1024, int(n)).tolist() for n in (17, 40)]

    def cfg(tp):
        c = _cfg(tp)
        c.model.quantization = QuantizationConfig(method="fp8_block")
        return c

    single = LLMEngine(cfg(1), model_config=mc)
    assert getattr(single.model, "fp8", False)
    ref = _run(single, prompts, n=5)
    launcher = TPEngineLauncher(cfg(2), model_config=mc, device_type="cpu")
    try:
        eng = launcher.engine()
        assert getattr(eng.model, "fp8", False)
        got = _run(eng, prompts, n=5)
    finally:
        launcher.shutdown()
    assert got == ref


@pytest.mark.timeout(300)
def test_pipelined_schedule_matches_sync_single_process_and_tp2():
    """Asynchronous (pipelined) scheduling forced on CPU engines: step n+1 is enqueued
    before step n's tokens are applied, pending decode inputs are scattered from the
    previous sample tensor -- on a TP2 engine rank 0 broadcasts that tensor and the
    worker repeats the scatter.  Greedy tokens equal the synchronous engine's."""
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (9, 40, 23, 3)]
    ref = _run(LLMEngine(_cfg(1), model_config=MC), prompts, n=7)
    single = LLMEngine(_cfg(1), model_config=MC)
    single._async = True
    assert _run(single, prompts, n=7) == ref
    launcher = TPEngineLauncher(_cfg(2), model_config=MC, device_type="cpu")
    try:
        eng = launcher.engine()
        eng._async = True
        got = _run(eng, prompts, n=7)
        again = _run(eng, prompts[:2], n=5)            # the pipeline drains and restarts cleanly
        broadcasts = eng.runner.broadcast_steps
    finally:
        launcher.shutdown()
    assert broadcasts > 0                              # decode inputs really came from the device
    assert got == ref
    assert again == [r[:5] for r in ref[:2]]


@pytest.mark.timeout(300)
def test_tp2_prefix_caching_matches_single_process():
    """Prompts sharing a long prefix on a TP2 engine with prefix caching: cached blocks
    are reused on every rank (the plan's block tables point at them), and the greedy
    tokens equal the single-process engine without caching."""
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(5)
    prefix = rng.integers(0, 1000, 64).tolist()
    prompts = [prefix + rng.integers(0, 1000, int(n)).tolist() for n in (5, 17, 9)]
    ref = _run(LLMEngine(_cfg(1), model_config=MC), prompts, n=6)
    cfg = _cfg(2)
    cfg.engine.enable_prefix_caching = True
    launcher = TPEngineLauncher(cfg, model_config=MC, device_type="cpu")
    try:
        eng = launcher.engine()
        first = _run(eng, prompts[:1], n=6)            # fills the cache with the prefix blocks
        rest = _run(eng, prompts[1:], n=6)
        hits = eng.bm.stats()["prefix_block_hits"]
    finally:
        launcher.shutdown()
    assert first + rest == ref
    assert hits > 0                                   # the later prompts reused the prefix blocks


@pytest.mark.timeout(600)
def test_worker_group_recovery_completes_every_request():
    """Failure injection on the host: a gloo TP2 engine's worker process is killed in the
    middle of serving.  The next step raises DistributedError; the launcher replaces the
    worker group (fresh processes and rendezvous, shards rebuilt), the engine re-queues
    every live sequence as a recompute preemption, and every request completes with the
    same greedy tokens as a single-process engine."""
    import os
    from rusteeze_b200.core.errors import DistributedError
    from rusteeze_b200.engine.llm_engine import LLMEngine
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (20, 33, 9, 40)]
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)

    def run(eng, kill=None):
        ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
        done, steps = {}, 0
        while eng.has_unfinished_requests():
            if kill is not None and steps == 4:
                kill()
                kill = None
            try:
                outs = eng.step()
            except DistributedError:
                eng.tp_launcher.recover()
                continue
            steps += 1
            for o in outs:
                if o.finished:
                    done[o.request_id] = o.outputs[0].token_ids
        return [done[i] for i in ids]

    ref = run(LLMEngine(_cfg(1), model_config=MC))
    os.environ["RZ_PG_TIMEOUT_S"] = "20"
    launcher = TPEngineLauncher(_cfg(2), model_config=MC, device_type="cpu")
    try:
        def kill():
            victim = launcher.procs[0]
            victim.kill()                   # our own child process, by handle
            victim.join(10)
        got = run(launcher.engine(), kill)
        assert launcher.recoveries == 1
        assert launcher.engine().stats_counters["worker_recoveries"] == 1
        assert got == ref
    finally:
        os.environ.pop("RZ_PG_TIMEOUT_S", None)
        launcher.shutdown(timeout=5.0)


def test_async_engine_recovers_from_a_dead_worker():
    """The serving loop: a DistributedError from a step triggers the engine's worker-group
    recovery (a stub launcher here), the stream continues, and the engine stays healthy."""
    import asyncio
    from rusteeze_b200.core.errors import DistributedError
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    from rusteeze_b200.engine.llm_engine import LLMEngine
    eng = LLMEngine(_cfg(1), model_config=MC)
    real_step = eng.step
    state = {"n": 0}

    def flaky_step():
        state["n"] += 1
        if state["n"] == 3:
            raise DistributedError("tensor-parallel worker rank(s) [1] exited")
        return real_step()

    class _Launcher:
        recoveries = 0

        def recover(self):
            self.recoveries += 1

    eng.step = flaky_step
    eng.tp_launcher = _Launcher()
    ae = AsyncLLMEngine(eng).start()
    try:
        async def go():
            out = None
            async for o in ae.generate(None, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True), "r",
                                       list(range(5, 30))):
                out = o
            return out
        out = asyncio.run(go())
        assert out.finished and len(out.outputs[0].token_ids) == 6
        assert eng.tp_launcher.recoveries == 1 and ae.healthy and ae.is_ready
    finally:
        ae.shutdown()


MC8 = ModelConfig(name="tp-tiny8", hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                  num_attention_heads=8, num_key_value_heads=4, vocab_size=1000, rms_norm_eps=1e-5,
                  max_position_embeddings=512)


@pytest.mark.timeout(600)
@pytest.mark.parametrize("world", [4, 8])
def test_tp4_tp8_gloo_match_single_process_sync_and_pipelined(world):
    """The host side of wider tensor parallelism: the plan ring with 3 or 7 readers, weights
    and vocabulary split 4 or 8 ways, kv heads split (4 kv heads at TP4) or replicated (TP8),
    and the pipelined schedule's device-to-device broadcast of the sampled tokens to every
    worker.  Greedy tokens equal the single-process engine's."""
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (33, 8, 61)]
    ref = _run(LLMEngine(_cfg(1), model_config=MC8), prompts, n=6)
    launcher = TPEngineLauncher(_cfg(world), model_config=MC8, device_type="cpu")
    try:
        eng = launcher.engine()
        got = _run(eng, prompts, n=6)
        eng._async = True
        piped = _run(eng, prompts, n=6)
    finally:
        launcher.shutdown()
    assert got == ref
    assert piped == ref


@pytest.mark.timeout(600)
def test_tp4_gloo_mixtral_expert_parallel_matches_single_process():
    from rusteeze_b200.models.config import ModelArchitecture
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    mc = ModelConfig(name="ep4-tiny", architecture=ModelArchitecture.MIXTRAL, hidden_size=128,
                     intermediate_size=192, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=4,
                     vocab_size=1000, rms_norm_eps=1e-5, max_position_embeddings=512, num_local_experts=8,
                     num_experts_per_tok=2)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (25, 50)]
    ref = _run(LLMEngine(_cfg(1), model_config=mc), prompts)
    launcher = TPEngineLauncher(_cfg(4), model_config=mc, device_type="cpu")
    try:
        got = _run(launcher.engine(), prompts)
    finally:
        launcher.shutdown()
    assert got == ref


@pytest.mark.timeout(300)
def test_tp2_alibi_slopes_follow_each_rank_s_heads():
    """ALiBi at TP2: every rank adds the slopes of its own query heads (a slice of the
    model's slopes); greedy tokens equal the single-process engine's."""
    import dataclasses
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    mc = dataclasses.replace(MC8, name="tp-alibi", position_embedding="alibi")
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (44, 13)]
    ref = _run(LLMEngine(_cfg(1), model_config=mc), prompts)
    launcher = TPEngineLauncher(_cfg(2), model_config=mc, device_type="cpu")
    try:
        got = _run(launcher.engine(), prompts)
    finally:
        launcher.shutdown()
    assert got == ref


@pytest.mark.timeout(300)
def test_tp2_prompt_logprobs_beam_search_guided_decoding_and_embeddings_match_single_process():
    """Host-side request features on a TP2 engine: prompt scoring (the executor's explicit
    forward), beam search (forked beams' block tables and copy-on-write copies reach the
    workers through the plans), guided decoding (rank 0's sampler masks the logits) and
    embeddings give what the single-process engine gives."""
    from rusteeze_b200.core.sampling_params import GuidedDecodingParams
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (40, 9)]
    reqs = [SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True, prompt_logprobs=2),
            SamplingParams(n=2, best_of=3, use_beam_search=True, temperature=0.0, max_tokens=6, ignore_eos=True),
            SamplingParams(temperature=0.0, max_tokens=12, guided_decoding=GuidedDecodingParams(regex=r"[a-f]{3,6}"))]

    def run(eng):
        ids = [eng.add_request(None, None, sp, p).request_id for sp in reqs for p in prompts]
        done = {}
        while eng.has_unfinished_requests():
            for o in eng.step():
                if o.finished:
                    done[o.request_id] = o
        return [done[i] for i in ids]

    single = LLMEngine(_cfg(1), model_config=MC)
    ref = run(single)
    ref_emb = single.embed(prompts, "last") + single.embed(prompts, "mean")
    launcher = TPEngineLauncher(_cfg(2), model_config=MC, device_type="cpu")
    try:
        got = run(launcher.engine())
        # embeddings: rank 0 returns hidden rows and still joins the LM head's all-gather
        emb = launcher.engine().embed(prompts, "last") + launcher.engine().embed(prompts, "mean")
    finally:
        launcher.shutdown()
    for a, b in zip(emb, ref_emb):
        assert np.abs(a - b).max() < 1e-4
    for a, b in zip(got, ref):
        assert [c.token_ids for c in a.outputs] == [c.token_ids for c in b.outputs]
        if b.prompt_logprobs is not None:
            assert len(a.prompt_logprobs) == len(b.prompt_logprobs)
            for x, y in zip(a.prompt_logprobs[1:], b.prompt_logprobs[1:]):
                assert x.keys() == y.keys() and max(abs(x[t] - y[t]) for t in x) < 1e-4
