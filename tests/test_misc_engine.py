"""Smaller engine components: batch-size SLO controller, memory report,
incremental detokenizer, chat templates, sampler host paths, abort/timeout."""
import time

import pytest

from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.batch_optimizer import BatchOptimizer, BatchOptimizerConfig
from rusteeze_b200.tokenizer.chat_template import ChatFormat, ChatTemplate
from rusteeze_b200.tokenizer.tokenizer import ByteTokenizer, IncrementalDetokenizer


def test_batch_optimizer_shrinks_and_grows():
    bo = BatchOptimizer(BatchOptimizerConfig(target_latency_s=0.05, max_batch=64, cooldown_steps=1))
    for _ in range(20):
        bo.observe(0.2)
    assert bo.batch < 64
    small = bo.batch
    for _ in range(60):
        bo.observe(0.005)
    assert bo.batch > small and bo.adjustments > 1


def test_incremental_detok_equals_full_decode():
    tok = ByteTokenizer()
    text = "héllo wörld — streaming ✓ text"
    ids = tok.encode(text, add_special_tokens=False)
    d = IncrementalDetokenizer(tok, [1])
    out = "".join(d.step(i) for i in ids)
    assert out == text == tok.decode(ids)


@pytest.mark.parametrize("fmt,needle", [(ChatFormat.LLAMA3, "<|start_header_id|>assistant"),
                                        (ChatFormat.CHATML, "<|im_start|>assistant"),
                                        (ChatFormat.LLAMA, "[INST] <<SYS>>"), (ChatFormat.PHI3, "<|assistant|>"),
                                        (ChatFormat.MISTRAL, "[INST] sys\n\nhi [/INST]")])
def test_chat_templates(fmt, needle):
    msgs = [{"role": "system", "content": "sys"}, {"role": "user", "content": "hi"}]
    assert needle in ChatTemplate(fmt).apply(msgs)
    assert ChatFormat.from_model_name("Meta-Llama-3-8B-Instruct") == ChatFormat.LLAMA3
    assert ChatFormat.from_model_name("unknown") == ChatFormat.CHATML


def test_jinja_template():
    t = ChatTemplate(jinja="{% for m in messages %}[{{ m.role }}]{{ m.content }}{% endfor %}"
                           "{% if add_generation_prompt %}[assistant]{% endif %}")
    assert t.apply([{"role": "user", "content": "x"}]) == "[user]x[assistant]"


def _tiny_engine(**kw):
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.engine.llm_engine import LLMEngine
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 64
    for k, v in kw.items():
        if k == "preemption_mode":
            cfg.engine.scheduling.preemption_mode = v
        else:
            setattr(cfg.engine, k, v)
    return LLMEngine(cfg)


def test_memory_report_and_host_sampling_paths():
    from rusteeze_b200.utils.memory import memory_report
    eng = _tiny_engine()
    rep = memory_report(eng)
    assert rep["kv_blocks"] == 64 and rep["weights_gib"] > 0
    params = [SamplingParams(temperature=1.0, mirostat_mode=2, max_tokens=4, ignore_eos=True, seed=1),
              SamplingParams(temperature=0.9, typical_p=0.5, max_tokens=4, ignore_eos=True, seed=2),
              SamplingParams(temperature=1.0, repetition_penalty=1.3, frequency_penalty=0.5, presence_penalty=0.2,
                             logit_bias={7: 5.0}, max_tokens=4, ignore_eos=True, seed=3, logprobs=3),
              SamplingParams(n=2, best_of=3, temperature=0.8, max_tokens=3, ignore_eos=True, seed=4)]
    ids = [eng.add_request(None, "hello there", p).request_id for p in params]
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o
    assert len(done[ids[2]].outputs[0].logprobs) == 4
    assert len(done[ids[3]].outputs) == 2            # best_of 3 -> n 2
    assert eng.bm.stats()["forks"] >= 2


def test_stop_strings_eos_and_min_tokens():
    eng = _tiny_engine()
    eos = eng.eos_ids[0]
    sp = SamplingParams(temperature=0.0, max_tokens=20, min_tokens=3, logit_bias={eos: 100.0})
    eng.add_request("a", None, sp, [5, 6, 7])
    out = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            out = o
    # EOS is forced by the bias but masked until min_tokens is reached
    assert len(out.outputs[0].token_ids) == 4 and out.outputs[0].finish_reason == "stop"


def test_abort_frees_blocks():
    eng = _tiny_engine()
    eng.add_request("x", None, SamplingParams(max_tokens=50, ignore_eos=True), list(range(40)))
    eng.step()
    assert eng.bm.num_free_gpu_blocks() < 64
    eng.abort_request("x")
    assert eng.bm.num_free_gpu_blocks() == 64 and not eng.has_unfinished_requests()


def test_async_engine_stall_watchdog_marks_not_ready_then_recovers():
    """A step that blocks (a stand-in for a collective waiting on a dead peer) makes the
    engine not ready after stall_timeout_s; when the step returns, readiness comes back."""
    import threading
    import time
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine

    class _StuckEngine:
        device = "cpu"

        def __init__(self):
            self.release = threading.Event()
            self.entered = threading.Event()
            self.pending = True

        def has_unfinished_requests(self):
            return self.pending

        def step(self):
            self.entered.set()
            self.release.wait(10.0)
            self.pending = False
            return []

        def abort_request(self, rid):
            pass

    stub = _StuckEngine()
    ae = AsyncLLMEngine(stub, stall_timeout_s=0.2).start()
    try:
        assert stub.entered.wait(5.0)
        time.sleep(0.4)
        assert not ae.is_ready and ae.healthy          # stalled, not failed
        stub.release.set()
        for _ in range(100):
            if ae.is_ready:
                break
            time.sleep(0.02)
        assert ae.is_ready
    finally:
        stub.release.set()
        ae.shutdown()


def test_closing_a_stream_aborts_the_request_in_the_engine():
    """A client that stops reading (SSE disconnect closes the async generator) must not
    leave its request generating: the engine drops it at its next loop iteration."""
    import asyncio
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    eng = _tiny_engine()
    ae = AsyncLLMEngine(eng).start()

    async def client():
        sp = SamplingParams(temperature=0.0, max_tokens=10_000, ignore_eos=True)
        gen = ae.generate(None, sp, "r-disconnect", prompt_token_ids=list(range(5, 25)))
        got = 0
        async for _ in gen:
            got += 1
            if got == 2:
                break
        await gen.aclose()
        for _ in range(200):                    # the loop stays alive while the engine drops it
            if not eng.has_unfinished_requests():
                break
            await asyncio.sleep(0.02)
        return got

    try:
        assert asyncio.run(client()) == 2
        assert not eng.has_unfinished_requests()
        assert eng.stats_counters["requests_aborted"] >= 1
        assert ae.healthy and ae._thread.is_alive()
    finally:
        ae.shutdown()


def test_a_vanished_client_loop_does_not_stop_the_engine_thread():
    """Outputs for a client whose event loop has closed are dropped and its request
    aborted; the engine thread keeps serving the next client."""
    import asyncio
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    eng = _tiny_engine()
    ae = AsyncLLMEngine(eng).start()

    async def first():
        sp = SamplingParams(temperature=0.0, max_tokens=10_000, ignore_eos=True)
        gen = ae.generate(None, sp, "r-gone", prompt_token_ids=list(range(5, 25)))
        async for _ in gen:
            return                              # the loop closes with the stream still open

    async def second():
        sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
        last = None
        async for out in ae.generate(None, sp, "r-next", prompt_token_ids=list(range(30, 40))):
            last = out
        return last

    try:
        asyncio.run(first())
        out = asyncio.run(second())
        assert out.finished and len(out.outputs[0].token_ids) == 4
        assert ae._thread.is_alive()
        for _ in range(200):
            if not eng.has_unfinished_requests():
                break
            time.sleep(0.02)
        assert not eng.has_unfinished_requests()
    finally:
        ae.shutdown()


@pytest.mark.parametrize("mode", ["recompute", "swap"])
def test_requests_larger_than_the_kv_cache_are_reported_not_stuck(mode):
    """A prompt that fits the model's context but not the whole KV cache (64 blocks of 16
    tokens here) finishes at once with finish_reason "length" instead of waiting forever;
    one that outgrows the cache while generating ends the same way (in swap mode it used
    to be swapped out and never fit back); other requests are unaffected."""
    eng = _tiny_engine(swap_space_gb=0.01, preemption_mode=mode)     # 64 GPU blocks = 1024 tokens of KV
    eng.add_request("big", None, SamplingParams(max_tokens=4, temperature=0.0), list(range(1100)))
    eng.add_request("grows", None, SamplingParams(max_tokens=200, temperature=0.0, ignore_eos=True),
                    list(range(900)))
    eng.add_request("small", None, SamplingParams(max_tokens=3, temperature=0.0, ignore_eos=True), list(range(20)))
    done = {}
    for _ in range(400):
        if not eng.has_unfinished_requests():
            break
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o.outputs[0]
    assert not eng.has_unfinished_requests()
    assert done["big"].finish_reason == "length" and done["big"].token_ids == []
    assert done["grows"].finish_reason == "length" and 0 < len(done["grows"].token_ids) < 200
    assert done["small"].finish_reason == "length" and len(done["small"].token_ids) == 3


@pytest.mark.parametrize("pipelined", [False, True])
def test_one_request_s_host_side_failure_ends_only_that_request(pipelined):
    """An exception in one request's post-processing (here injected into its stop check)
    aborts that request with the error as its stop reason; the batch's other requests
    finish with the tokens they would have had, and the engine keeps serving."""
    import numpy as np
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.engine.llm_engine import LLMEngine

    def make():
        cfg = Config()
        cfg.model.preset, cfg.model.device, cfg.model.dtype = "tiny-llama", "cpu", "float32"
        cfg.engine.num_gpu_blocks = 64
        eng = LLMEngine(cfg)
        eng._async = pipelined
        return eng

    rng = np.random.default_rng(0)
    prompts = {f"r{i}": rng.integers(3, 200, 20).tolist() for i in range(3)}
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)

    def run(eng):
        for rid, p in prompts.items():
            eng.add_request(rid, None, sp, p)
        done = {}
        while eng.has_unfinished_requests():
            for o in eng.step():
                if o.finished:
                    done[o.request_id] = o.outputs[0]
        return done

    ref = run(make())
    eng = make()
    real = eng._check_stop

    def flaky(s, tok):
        if s.request.request_id == "r1" and s.num_generated == 3:
            raise RuntimeError("injected post-processing failure")
        return real(s, tok)
    eng._check_stop = flaky
    got = run(eng)
    assert got["r1"].finish_reason == "abort" and "injected" in got["r1"].stop_reason
    for rid in ("r0", "r2"):
        assert got[rid].token_ids == ref[rid].token_ids and got[rid].finish_reason == "length"
    assert eng.stats_counters["requests_failed"] == 1
    assert eng.bm.num_free_gpu_blocks() == eng.bm.num_gpu_blocks
    eng._check_stop = real
    assert run(eng)["r0"].token_ids == ref["r0"].token_ids     # still serving


def test_a_failed_request_is_counted_as_an_error_in_the_metrics():
    from rusteeze_b200.core.outputs import CompletionOutput, RequestOutput
    from rusteeze_b200.metrics.registry import EngineMetrics
    m = EngineMetrics(model_name="m")
    bad = RequestOutput("r", None, [1], [CompletionOutput(0, "", [], finish_reason="abort",
                                                          stop_reason="error: RuntimeError('x')")], True)
    m.on_request_finished(bad, "completions")
    text = m.export().decode()
    assert 'errors_total{type="request_failed"} 1.0' in text
    assert any('status="error"' in ln and ln.rstrip().endswith(" 1.0") for ln in text.splitlines()
               if "requests_total" in ln)
