"""Stop strings and streaming (CPU): the engine's stop check and streamed deltas, driven
with chosen tokens (a byte tokenizer).  A stop string split over several tokens is never streamed, not
even its beginning, while text that only looked like the start of one is released once
it is clear; the concatenated deltas equal the final text in every case."""
import pytest

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig

BYTES = ModelConfig(name="tiny-bytes", hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                    num_attention_heads=2, num_key_value_heads=1, vocab_size=256, max_position_embeddings=512)


def _engine():
    cfg = Config()
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 32
    return LLMEngine(cfg, model_config=BYTES)


def _drive(eng, text, **sp):
    req = eng.add_request(None, None, SamplingParams(max_tokens=100, ignore_eos=True, **sp), [65, 66, 67])
    s = req.seqs[0]
    streamed = []
    for b in eng.tokenizer.encode(text, add_special_tokens=False):
        s.append_token(b)
        eng._check_stop(s, b)
        streamed.append(req.to_output(delta=True).delta_text[0])
        if s.is_finished():
            break
    return "".join(streamed), s.output_text, s.finish_reason


@pytest.mark.parametrize("text,stops,final", [
    ("hello ENDworld", ["END"], "hello "),            # stop split over three tokens
    ("an ENvelope END", ["END"], "an ENvelope "),     # a partial match that was not a stop
    ("abcab!", ["abd", "cab!"], "ab"),                # overlapping candidates
    ("x<|eot|>y", ["<|eot|>"], "x"),
])
def test_streamed_text_never_contains_a_stop_string(text, stops, final):
    streamed, out, reason = _drive(_engine(), text, stop=stops)
    assert out == final and reason == "stop"
    assert streamed == final


def test_stop_string_kept_when_asked():
    streamed, out, reason = _drive(_engine(), "hello ENDworld", stop=["END"], include_stop_str_in_output=True)
    assert out == "hello END" and streamed == "hello END" and reason == "stop"


def test_text_without_stop_streams_completely():
    eng = _engine()
    req = eng.add_request(None, None, SamplingParams(max_tokens=5, ignore_eos=True, stop=["zz"]), [65])
    s = req.seqs[0]
    streamed = []
    for b in eng.tokenizer.encode("abcdz", add_special_tokens=False):
        s.append_token(b)
        eng._check_stop(s, b)
        streamed.append(req.to_output(delta=True).delta_text[0])
    assert s.finish_reason == "length"
    assert "".join(streamed) == s.output_text == "abcdz"     # the held-back "z" is released at the end
