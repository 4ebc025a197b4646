"""Guided (structured) decoding: the regex automaton against Python's `re` (full matches)
and the `regex` module (partial matches: a prefix keeps the automaton alive exactly when
it can still be completed), JSON Schema compilation against instances, token masks
against a brute-force check of every token, and constrained generation through the
engine and the HTTP API with random weights: every output satisfies its constraint."""
import json
import re

import numpy as np
import pytest
import regex as regex_mod
from hypothesis import given, settings, strategies as st

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.errors import InvalidRequestError
from rusteeze_b200.core.sampling_params import GuidedDecodingParams, SamplingParams
from rusteeze_b200.engine.guided.guide import TokenIndex, fsm_for
from rusteeze_b200.engine.guided.json_schema import any_object, schema_to_regex
from rusteeze_b200.engine.guided.regex_fsm import RegexError, RegexFSM
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.tokenizer.tokenizer import ByteTokenizer

PATTERNS = [r"[0-9]{3}-[a-c]+", r"(ab|ba)*c?", r"a{2,4}b{0,2}", r"(x|yz)+(\.[xy]{1,2})?", r"[^abc]b*",
            r"\d\w\s?", r"(?:a|b)(?P<n>c|d)e?", r"a.c", r"[a-c-]+", r"^ab+$"]
ALPHA = "abcxyz0123-. \n"


@settings(max_examples=400, deadline=None, derandomize=True)
@given(st.sampled_from(PATTERNS), st.text(alphabet=ALPHA, max_size=8))
def test_fsm_matches_python_re_and_partial_matches(pat, s):
    f = fsm_for(pat)
    assert f.fullmatch(s) == bool(re.fullmatch(pat, s))
    alive = f.walk(f.start, s) >= 0
    assert alive == (regex_mod.fullmatch(pat, s, partial=True) is not None)


def _regex_strategy():
    """Random patterns over a small alphabet: literals, escapes, classes (negated, ranges),
    dots, groups, alternation and every quantifier form, nested."""
    atoms = st.sampled_from(["a", "b", "c", "-", r"\.", r"\d", r"\w", r"\s", ".", "[ab]", "[^a]", "[a-c]",
                             "[0-9x]", r"[\d.]", "1"])

    def extend(inner):
        quant = st.sampled_from(["*", "+", "?", "{2}", "{0,2}", "{1,}", "*?", "{1,3}"])
        return st.one_of(
            st.tuples(inner, quant).map(lambda t: f"(?:{t[0]}){t[1]}"),
            st.lists(inner, min_size=2, max_size=3).map("".join),
            st.lists(inner, min_size=2, max_size=3).map(lambda xs: "(" + "|".join(xs) + ")"),
        )
    return st.recursive(atoms, extend, max_leaves=8)


@settings(max_examples=300, deadline=None, derandomize=True)
@given(_regex_strategy(), st.lists(st.text(alphabet="abc1x-. ", max_size=7), min_size=1, max_size=6))
def test_random_patterns_match_python_re(pat, strings):
    f = RegexFSM(pat)
    # the regex module's partial matching mishandles lazy quantifiers ("(?:a)*?a" takes
    # "a1" as a partial match); lazy and greedy forms define the same language
    greedy = pat.replace("*?", "*")
    for s in strings:
        assert f.fullmatch(s) == bool(re.fullmatch(pat, s)), (pat, s)
        alive = f.walk(f.start, s) >= 0
        assert alive == (regex_mod.fullmatch(greedy, s, partial=True) is not None), (pat, s)


def test_empty_patterns_match_only_the_empty_string():
    for p in ("", "()", "(|a)b?"):
        f = RegexFSM(p)
        assert f.fullmatch("") and not f.fullmatch("c")
    for bad in ({"enum": []}, {"anyOf": []}, {"oneOf": "x"}):
        with pytest.raises(ValueError):
            schema_to_regex(bad)


def test_unsupported_patterns_are_refused():
    for p in (r"(a)\1", r"(?=a)b", r"a{5,2}", "[abc", "(ab", "*a"):
        with pytest.raises(RegexError):
            RegexFSM(p)


SCHEMA = {"type": "object",
          "properties": {"name": {"type": "string", "maxLength": 6},
                         "age": {"type": "integer"},
                         "tags": {"type": "array", "items": {"enum": ["a", "b"]}, "maxItems": 2},
                         "kind": {"$ref": "#/$defs/kind"},
                         "score": {"type": ["number", "null"]}},
          "required": ["name", "age"],
          "$defs": {"kind": {"enum": ["x", "y"]}}}


def _valid(d) -> bool:
    if not isinstance(d, dict) or set(d) - set(SCHEMA["properties"]) or not {"name", "age"} <= set(d):
        return False
    if not (isinstance(d["name"], str) and len(d["name"]) <= 6) or type(d["age"]) is not int:
        return False
    if "tags" in d and not (isinstance(d["tags"], list) and len(d["tags"]) <= 2 and set(d["tags"]) <= {"a", "b"}):
        return False
    if "kind" in d and d["kind"] not in ("x", "y"):
        return False
    return "score" not in d or d["score"] is None or type(d["score"]) in (int, float)


def test_schema_regex_accepts_instances_and_rejects_others():
    f = RegexFSM(schema_to_regex(SCHEMA))
    good = [{"name": "bo", "age": 3}, {"name": "", "age": -12, "tags": ["a", "b"], "kind": "y", "score": 1.5},
            {"name": "ab\"c", "age": 0, "score": None}, {"name": "x", "age": 7, "kind": "x"}]
    for d in good:
        assert _valid(d)
        for sep in ((",", ":"), (", ", ": ")):
            assert f.fullmatch(json.dumps(d, separators=sep)), d
    bad = ['{"age": 3}', '{"name": "toolongname", "age": 3}', '{"name": "a", "age": 1.5}',
           '{"name": "a", "age": 1, "tags": ["c"]}', '{"name": "a", "age": 1, "extra": 1}',
           '{"age": 1, "name": "a"}']                     # properties come in the schema's order
    for t in bad:
        assert not f.fullmatch(t), t
    assert RegexFSM(any_object()).fullmatch('{"a": [1, {"b": null}], "c": "x"}')


def _conforms(v, sch, root):
    """The schema subset the compiler supports, checked on a parsed value."""
    if "$ref" in sch:
        node = root
        for part in sch["$ref"][2:].split("/"):
            node = node[part]
        return _conforms(v, node, root)
    if "const" in sch:
        return v == sch["const"]
    if "enum" in sch:
        return v in sch["enum"]
    for k in ("anyOf", "oneOf"):
        if k in sch:
            return any(_conforms(v, x, root) for x in sch[k])
    t = sch.get("type")
    if isinstance(t, list):
        return any(_conforms(v, dict(sch, type=x), root) for x in t)
    if t == "string":
        return isinstance(v, str) and len(v) <= sch.get("maxLength", 10 ** 9) and len(v) >= sch.get("minLength", 0)
    if t == "integer":
        return type(v) is int
    if t == "number":
        return type(v) in (int, float)
    if t == "boolean":
        return type(v) is bool
    if t == "null":
        return v is None
    if t == "array":
        return (isinstance(v, list) and sch.get("minItems", 0) <= len(v) <= sch.get("maxItems", 10 ** 9)
                and all(_conforms(x, sch.get("items", {}), root) for x in v))
    if t == "object":
        props = sch.get("properties", {})
        return (isinstance(v, dict) and set(v) <= set(props) and set(sch.get("required", [])) <= set(v)
                and all(_conforms(v[k], props[k], root) for k in v))
    return True


_SCHEMAS = [
    SCHEMA,
    {"type": "object", "properties": {"s": {"type": "string"}, "n": {"type": "number"},
                                      "o": {"type": "object", "properties": {"x": {"type": "null"}}}},
     "required": ["s"]},
    {"type": "array", "items": {"anyOf": [{"type": "integer"}, {"const": "k"}]}, "minItems": 1, "maxItems": 3},
    {"type": "object", "properties": {"a": {"type": "boolean"}, "b": {"enum": [1, "two", None]}}},
]


@pytest.mark.parametrize("i", range(len(_SCHEMAS)))
def test_every_string_of_a_schema_regex_is_conforming_json(i):
    sch = _SCHEMAS[i]
    pat = schema_to_regex(sch)

    @settings(max_examples=150, deadline=None, derandomize=True)
    @given(st.from_regex(pat, fullmatch=True))
    def check(text):
        assert _conforms(json.loads(text), sch, sch), text
    check()


def test_token_masks_equal_a_brute_force_check():
    tok = ByteTokenizer(300)
    ix = TokenIndex(tok, 300)
    f = fsm_for(r'"[a-c]{0,3}"|[0-9]+')
    rng = np.random.default_rng(0)
    states = {f.start}
    for s in ('"', '"ab', '"abc', "12", '"abc"'):
        states.add(f.walk(f.start, s))
    for _ in range(5):
        states.add(f.walk(f.start, "".join(rng.choice(list('"abc0123'), 2))))
    for stt in states:
        if stt < 0:
            continue
        m = ix.allowed(f, stt)
        want = np.array([bool(t) and f.walk(stt, t) >= 0 for t in ix.texts])
        assert (m == want).all()


class _PieceTokenizer:
    """SentencePiece-style: "▁" marks a word start and is a space, except at the very start
    of a decoded sequence, where it is dropped."""
    PIECES = ["<s>", "</s>", "a", "▁a", "b", "▁b", "▁", "1", "▁1", "-"]

    def encode(self, text, add_special_tokens=True):
        return [self.PIECES.index(text)] if text in self.PIECES else []

    def decode(self, ids, skip=True):
        s = "".join(self.PIECES[i] for i in ids if not (skip and i < 2)).replace("▁", " ")
        return s[1:] if s.startswith(" ") else s


def test_token_texts_keep_sentencepiece_leading_spaces():
    ix = TokenIndex(_PieceTokenizer(), len(_PieceTokenizer.PIECES))
    assert ix.texts[:6] == ["", "", "a", " a", "b", " b"]
    f = fsm_for("[ab]+")                            # words without spaces: "▁a" must be refused
    m = ix.allowed(f, f.start)
    assert m[2] and m[4] and not m[3] and not m[5]


class _WordTokenizer:
    """A large synthetic vocabulary (multi-character tokens), to reach the self-loop path."""

    def __init__(self, n, seed=0):
        rng = np.random.default_rng(seed)
        alpha = list('abcdefxyz0123456789 .,:"{}[]-\\')
        self.t = ["".join(rng.choice(alpha, int(rng.integers(1, 6)))) for _ in range(n)]

    def decode(self, ids, skip=True):
        return "".join(self.t[i] for i in ids)


def test_large_vocabulary_masks_equal_a_brute_force_check():
    ix = TokenIndex(_WordTokenizer(6000), 6000)
    f = fsm_for(any_object())
    for text in ("", "{", '{"a', '{"a\\', '{"ab": "x y', '{"a": [1, 2', '{"a": {"b": 1}'):
        stt = f.walk(f.start, text)
        assert stt >= 0
        m = ix.allowed(f, stt)
        want = np.array([bool(t) and f.walk(stt, t) >= 0 for t in ix.texts])
        assert (m == want).all(), text


def _engine(preset="tiny-llama"):
    cfg = Config()
    cfg.model.preset, cfg.model.device, cfg.model.dtype = preset, "cpu", "float32"
    cfg.engine.num_gpu_blocks = 128
    cfg.engine.max_num_seqs = 8
    return LLMEngine(cfg)


def _gen(eng, g, n=1, temp=0.9, max_tokens=80, seed=1, **kw):
    eng.add_request(None, "hello", SamplingParams(n=n, temperature=temp, max_tokens=max_tokens, guided_decoding=g,
                                                  seed=seed, **kw))
    fin = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                fin = o
    return fin.outputs


@pytest.fixture(scope="module")
def eng():
    return _engine()


def test_choice_regex_and_schema_outputs_satisfy_their_constraints(eng):
    for seed in range(3):
        outs = _gen(eng, GuidedDecodingParams(choice=["yes", "no", "maybe not"]), n=3, seed=seed)
        assert all(o.text in ("yes", "no", "maybe not") and o.finish_reason == "stop" for o in outs)
        outs = _gen(eng, GuidedDecodingParams(regex=r"[0-9]{3}-[a-z]{2,5}"), n=2, seed=seed)
        assert all(re.fullmatch(r"[0-9]{3}-[a-z]{2,5}", o.text) for o in outs)
        outs = _gen(eng, GuidedDecodingParams(json_schema=SCHEMA), max_tokens=200, seed=seed,
                    logit_bias={ord("}") + 3: 4.0, ord(",") + 3: 2.0, ord('"') + 3: 3.0})
        for o in outs:
            assert o.finish_reason == "stop", o.text
            assert _valid(json.loads(o.text)), o.text
    greedy = _gen(eng, GuidedDecodingParams(regex=r"(ab|cd){2}x?"), temp=0.0)
    assert re.fullmatch(r"(ab|cd){2}x?", greedy[0].text)


def test_top_k_applies_to_the_constrained_distribution(eng):
    """Guided rows are sampled on the host: top_k=1 at temperature 1 must give the greedy
    constrained output whatever the seed."""
    g = GuidedDecodingParams(regex=r"[a-z]{4}")
    greedy = _gen(eng, g, temp=0.0)[0].text
    assert {_gen(eng, g, temp=1.0, top_k=1, seed=s)[0].text for s in range(4)} == {greedy}
    assert len({_gen(eng, g, temp=1.0, seed=s)[0].text for s in range(4)}) > 1


def test_json_object_mode_prefixes_stay_valid(eng):
    f = fsm_for(any_object())
    for seed in range(3):
        o = _gen(eng, GuidedDecodingParams(json_object=True), max_tokens=120, seed=seed,
                 logit_bias={ord("}") + 3: 6.0, ord("]") + 3: 4.0, ord('"') + 3: 3.0})[0]
        assert f.walk(f.start, o.text) >= 0, o.text
        if o.finish_reason == "stop":
            assert isinstance(json.loads(o.text), dict)


def test_ignore_eos_stops_when_the_constraint_is_complete(eng):
    outs = _gen(eng, GuidedDecodingParams(choice=["alpha", "beta"]), n=2, ignore_eos=True)
    assert all(o.text in ("alpha", "beta") and o.finish_reason == "stop" for o in outs)


def test_a_pattern_the_vocabulary_cannot_spell_ends_the_request(eng):
    """The byte tokenizer has no whole-character token for "é" (two UTF-8 bytes): after
    "ab" nothing can continue, so the request ends there instead of leaving the pattern."""
    for ignore_eos in (False, True):
        o = _gen(eng, GuidedDecodingParams(regex="abé+"), temp=0.0, ignore_eos=ignore_eos)[0]
        assert o.text == "ab" and o.finish_reason == "stop"


def test_invalid_constraints_are_refused(eng):
    for g in (GuidedDecodingParams(), GuidedDecodingParams(regex="a", choice=["a"]),
              GuidedDecodingParams(grammar="root ::= 'a'"), GuidedDecodingParams(regex="(a"),
              # malformed or unsupported schemas are the client's error, never a server one
              GuidedDecodingParams(json_schema={"properties": 7}), GuidedDecodingParams(json_schema={"$ref": 5}),
              GuidedDecodingParams(json_schema={"type": "string", "maxLength": 5000}),
              GuidedDecodingParams(json_schema={"type": "array", "maxItems": {"a": 1}})):
        with pytest.raises(InvalidRequestError):
            eng.add_request(None, "x", SamplingParams(guided_decoding=g))
    with pytest.raises(InvalidRequestError):
        eng.add_request(None, "x", SamplingParams(best_of=2, use_beam_search=True, temperature=0.0,
                                                  guided_decoding=GuidedDecodingParams(regex="a+")))


def test_structured_output_through_the_api():
    from fastapi.testclient import TestClient

    from rusteeze_b200.api.server import create_app
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    cfg = Config()
    cfg.logging.request_logging = False
    ae = AsyncLLMEngine(_engine()).start()
    try:
        c = TestClient(create_app(ae, cfg))
        schema = {"type": "object", "properties": {"ok": {"type": "boolean"}, "n": {"type": "integer"}},
                  "required": ["ok", "n"]}
        r = c.post("/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "answer in JSON"}], "max_tokens": 60, "temperature": 0.7,
            "seed": 4, "logit_bias": {str(ord("}") + 3): 5.0},
            "response_format": {"type": "json_schema", "json_schema": {"name": "a", "schema": schema}}})
        assert r.status_code == 200, r.text
        d = json.loads(r.json()["choices"][0]["message"]["content"])
        assert type(d["ok"]) is bool and type(d["n"]) is int
        r = c.post("/v1/completions", json={"prompt": "pick", "max_tokens": 10, "n": 3, "temperature": 1.0,
                                            "guided_choice": ["red", "green"]})
        assert r.status_code == 200 and {x["text"] for x in r.json()["choices"]} <= {"red", "green"}
        r = c.post("/v1/completions", json={"prompt": "x", "guided_regex": "(a"})
        assert r.status_code == 400
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                 "response_format": {"type": "xml"}})
        assert r.status_code == 400
    finally:
        ae.shutdown()
