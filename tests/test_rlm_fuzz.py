"""RLM environment fuzzing: the model's output is untrusted text, so random operation
lines (odd argument counts, negative and huge numbers, unknown variables, invalid and
catastrophically backtracking regexes) must always give a result or an error message
back to the model -- never an exception, never a stalled engine -- and whole RLM
sessions driven by a random model end within their iteration limit."""
import random
import time

import pytest

from rusteeze_b200.rlm.prompt_env import EnvLimits, ExecResult, PromptEnvironment, model_regex, parse_model_output
from rusteeze_b200.rlm.recursive_engine import MockInferenceModel, RecursiveEngine, RLMConfig

_ARGS = ["0", "-5", "10", "99999999999999999999", "__prompt__", "__chunks__", "x", "missing", "", "'q'",
         "(a+)+$", "a*a*b", "[unclosed", "\\w+\\s+\\w+", "(a)\\1", "split(,)", "join", "filter(a)", "sort",
         "count", "truncate(3)", "grep(a*a*b)", "grep(b.)", "map_subcall(sum)", "reduce(join)", "nope(1)"]
_OPS = ["FINAL", "FINAL_VAR", "PEEK", "DECOMPOSE", "SEARCH", "REGEX_SEARCH", "SET_VAR", "GET_VAR", "SUBCALL",
        "SUBCALL_VAR", "BATCH_SUBCALL", "TRANSFORM", "THINK", "final", "Peek"]


def _line(rng):
    op = rng.choice(_OPS)
    args = ", ".join(rng.choice(_ARGS) for _ in range(rng.randint(0, 4)))
    close = ")" if rng.random() < 0.9 else ""
    return f"{op}({args}{close}"


def _output(rng):
    return "\n".join(rng.choice([_line(rng), "thinking about it", "", "(((", "FINAL"]) for _ in range(3))


@pytest.mark.parametrize("seed", range(5))
def test_random_operations_never_raise_or_stall(seed):
    rng = random.Random(seed)
    prompt = "".join(rng.choice(["a", "b", " ", "\n", "é", "字", ". "]) for _ in range(20000))
    env = PromptEnvironment(prompt, EnvLimits(max_subcalls=50))
    env.store.set("x", ["a", "b", "c"])
    for _ in range(120):
        op = parse_model_output(_output(rng))
        t0 = time.monotonic()
        res = env.execute(op)
        assert isinstance(res, ExecResult)
        assert time.monotonic() - t0 < 10, op          # a model-written regex is bounded in time
        if res.subcalls:
            for sc in res.subcalls:
                env.store_subcall_result(sc, "r")
            if res.batch_target:
                env.store_batch_results(res.batch_target, ["r"] * len(res.subcalls))
        assert env.subcalls_made <= env.limits.max_subcalls


def test_a_catastrophic_pattern_falls_back_to_a_substring_match():
    text = "a" * 30000 + "needle"
    t0 = time.monotonic()
    assert model_regex("a*a*b", text, 0) is None                   # timed out in the child
    assert time.monotonic() - t0 < 6
    env = PromptEnvironment(text)
    res = env.execute(parse_model_output("SEARCH(a*a*z)"))
    assert res.error is None and res.stdout.startswith("0 match")  # no such substring
    assert model_regex("ne+dle", text, 0) == [(30000, "needle")]
    assert model_regex("needle", text, 0) == [(30000, "needle")]   # no repetition: in process


@pytest.mark.parametrize("seed", range(4))
def test_sessions_driven_by_a_random_model_end(seed):
    rng = random.Random(seed)

    def respond(_prompt):
        return _output(rng)
    model = MockInferenceModel(rules=[("", respond)])
    eng = RecursiveEngine(model, RLMConfig(max_iterations=12, max_depth=2, max_subcalls=40))
    r = eng.process("some long text " * 200, "summarise")
    assert r.stats.iterations <= 12
    assert isinstance(r.text, str)
