"""RLM tier: operation parsing, variable store, chunking, call tree, and the
full recursive loop driven by a keyword mock model and by the tiny CPU engine."""
import pytest

from rusteeze_b200.core.errors import InvalidRequestError
from rusteeze_b200.rlm import (MockInferenceModel, PromptEnvironment, RecursiveEngine, RecursiveScheduler,
                               RLMConfig, SchedulerLimits, VariableStore, adaptive_chunk, parse_model_output)
from rusteeze_b200.rlm.prompt_env import EnvLimits, utf8_slice
from rusteeze_b200.rlm.recursive_scheduler import CallState


def test_parse_ops():
    assert parse_model_output("Let me look.\nPEEK(0, 100)").kind == "PEEK"
    assert parse_model_output("peek(5,9)").args == (5, 9)
    assert parse_model_output('final("the answer")').args == ("the answer",)
    assert parse_model_output("FINAL_VAR(x)").kind == "FINAL_VAR"
    assert parse_model_output("SUBCALL_VAR(doc, summarize it, briefly)").args == ("doc", "summarize it, briefly")
    assert parse_model_output("DECOMPOSE(500)").args == (500, 200)
    assert parse_model_output("TRANSFORM(a, b, split(,))").args == ("a", "b", "split(,)")
    assert parse_model_output("regex_search(fo+)").kind == "SEARCH"
    t = parse_model_output("I am thinking about this")
    assert t.kind == "THINK"


def test_variable_store():
    st = VariableStore(memory_limit=1000)
    st.set("t", "hello world")
    st.set("l", ["a", "b"])
    st.set("k", [1, 2, 3])
    assert st.meta("t").type == "text" and st.meta("l").type == "list" and st.meta("k").type == "tokens"
    assert "t: text (11 chars)" in st.metadata_block()
    with pytest.raises(InvalidRequestError):
        st.set("big", "x" * 2000)
    assert not st.is_terminated()
    st.set_final_var("t")
    assert st.final_value() == "hello world"


def test_adaptive_chunk_boundaries_and_coverage():
    text = ("Sentence number %d is here. " * 200) % tuple(range(200))
    chunks = adaptive_chunk(text, 500, 50)
    assert all(len(c) <= 500 for c in chunks)
    assert chunks[0].endswith(". ")
    # every character is covered, in order
    joined_start = 0
    for c in chunks:
        i = text.find(c, max(0, joined_start - 60))
        assert i >= 0
        joined_start = i + len(c)
    assert joined_start == len(text)
    assert adaptive_chunk("short", 100, 10) == ["short"]


def test_utf8_safe_peek():
    s = "héllo wörld ✓"
    assert utf8_slice(s, 0, 2) == "h"          # cuts inside é -> dropped
    assert "✓" in utf8_slice(s, 0, 100)


def test_env_ops_and_limits():
    env = PromptEnvironment("alpha beta\ngamma alpha\ndelta", EnvLimits(max_subcalls=2))
    r = env.execute(parse_model_output("SEARCH(alp.a)"))
    assert r.stdout.startswith("2 match")
    env.execute(parse_model_output("SET_VAR(x, a,b,c)"))
    env.execute(parse_model_output("TRANSFORM(x, y, split(,))"))
    assert env.store.get("y") == ["a", "b", "c"]
    env.execute(parse_model_output("TRANSFORM(y, n, count)"))
    assert env.store.get("n") == 3
    r = env.execute(parse_model_output("BATCH_SUBCALL(y, do it)"))
    assert r.error and "limit" in r.error
    assert env.execute(parse_model_output("GET_VAR(nope)")).error


def _mock_pipeline(prompt_text):
    def root(prompt):
        if "__chunks____results" in prompt and "joined" in prompt:
            return "FINAL_VAR(joined)"
        if "__chunks____results" in prompt:
            return "TRANSFORM(__chunks____results, joined, join( | ))"
        if "__chunks__: list" in prompt:
            return "BATCH_SUBCALL(__chunks__, ZZSUMMARIZE)"
        return "DECOMPOSE(300, 20)"
    return MockInferenceModel([("ZZSUMMARIZE", "summary"), ("REPL over a long prompt", root)])


def test_rlm_end_to_end_with_mock():
    text = "\n\n".join(f"Paragraph {i}: " + "lorem ipsum " * 20 for i in range(6))
    model = _mock_pipeline(text)
    eng = RecursiveEngine(model, RLMConfig(max_iterations=10))
    res = eng.process(text, "summarize the document")
    assert res.terminated
    parts = res.text.split(" | ")
    assert parts and all(p == "summary" for p in parts)
    assert len(parts) > 1
    assert max(model.batch_sizes) == len(parts)        # all chunks submitted together
    assert res.stats.subcalls == len(parts) and res.cost_usd > 0
    assert eng.global_stats["sessions"] == 1


def test_rlm_auto_decompose_and_iteration_limit():
    text = "x" * 250_000
    model = MockInferenceModel(default="hmm, thinking")
    res = RecursiveEngine(model, RLMConfig(max_iterations=3)).process(text)
    assert res.stats.auto_decomposed and not res.terminated and res.stats.iterations == 3


def test_rlm_auto_resolve_mock():
    res = RecursiveEngine(MockInferenceModel(auto_resolve=2), RLMConfig()).process("short prompt")
    assert res.terminated and res.text == "auto-resolved" and res.stats.iterations == 2


def test_recursive_scheduler_tree():
    s = RecursiveScheduler(SchedulerLimits(max_depth=2, per_level_concurrency=2))
    a = s.spawn(0, "p", "i")
    b = s.spawn(a, "p", "i")
    with pytest.raises(RecursionError):
        s.spawn(b, "p", "i")
    c1, c2, c3 = s.spawn_batch(0, [("x", "y")] * 3)
    ready = s.ready()
    assert len([n for n in ready if n.depth == 1]) == 2      # per-level concurrency
    s.start(a)
    s.fail(a, "boom")
    assert s.nodes[b].state == CallState.CANCELLED            # cascade
    s.start(c1)
    assert s.check_timeouts(now=s.nodes[c1].started + 1e6) == [c1]
    s.complete(c2, "ok")
    assert s.nodes[c2].result == "ok"


def test_rlm_over_tiny_cpu_engine():
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.engine.llm_engine import LLMEngine
    from rusteeze_b200.rlm import EngineInferenceModel
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.model.max_model_len = 1024
    cfg.engine.num_gpu_blocks = 256
    cfg.engine.max_num_batched_tokens = 2048
    cfg.engine.enable_chunked_prefill = True
    eng = LLMEngine(cfg)
    m = EngineInferenceModel(eng)
    outs = m.infer_batch(["hello", "world", "again"], 4)
    assert len(outs) == 3 and all(o.completion_tokens >= 1 for o in outs)
    res = RecursiveEngine(m, RLMConfig(max_iterations=2, root_max_tokens=8)).process("some long text " * 20)
    assert res.stats.iterations == 2


from hypothesis import given, settings, strategies as st  # noqa: E402

from rusteeze_b200.rlm.prompt_env import OP_PATTERN, parse_model_output  # noqa: E402


@settings(max_examples=300, deadline=None, derandomize=True)
@given(st.from_regex(OP_PATTERN, fullmatch=True))
def test_every_string_of_the_operation_pattern_parses_to_an_operation(s):
    assert parse_model_output(s).kind != "THINK", s


def test_constrained_root_turns_are_operations():
    """With random weights, the orchestrator's turns (guided by the operation pattern) are
    operation lines or prefixes of one cut by max_tokens -- never free text."""
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.engine.guided import fsm_for
    from rusteeze_b200.engine.llm_engine import LLMEngine
    from rusteeze_b200.rlm import EngineInferenceModel
    cfg = Config()
    cfg.model.preset, cfg.model.device, cfg.model.dtype = "tiny-llama", "cpu", "float32"
    cfg.model.max_model_len = 2048
    cfg.engine.num_gpu_blocks = 256
    cfg.engine.max_num_batched_tokens = 2048
    cfg.engine.enable_chunked_prefill = True
    m = EngineInferenceModel(LLMEngine(cfg), temperature=0.8)
    f = fsm_for(OP_PATTERN)
    for prompt in ("task one", "task two", "task three"):
        out = m.infer(prompt, 60, pattern=OP_PATTERN).text
        assert f.walk(f.start, out) >= 0, out
    res = RecursiveEngine(m, RLMConfig(max_iterations=3, root_max_tokens=60)).process("some long text " * 20)
    assert res.stats.iterations >= 1
