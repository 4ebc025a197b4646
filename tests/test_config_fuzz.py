"""Config files with random malformed content (wrong types, nulls, lists where a
section belongs, unparsable text) are refused with a ConfigError that names the
problem -- never another exception -- and valid values of the wrong textual form
(numbers as strings, as environment variables give them) are accepted."""
import dataclasses
import random

import pytest

from rusteeze_b200.config.config import Config
from rusteeze_b200.config.loader import ConfigLoader
from rusteeze_b200.core.errors import ConfigError

_JUNK = [None, True, "abc", "", "12", "1e3", "0.5", -1, 0, 3, 1.5, 1e309, [1], [], {}, {"x": 1}, ".nan"]


def _fields(obj, prefix=()):
    for f in dataclasses.fields(obj):
        v = getattr(obj, f.name)
        if dataclasses.is_dataclass(v):
            yield from _fields(v, prefix + (f.name,))
        else:
            yield prefix + (f.name,)


def _nested(path, value):
    d = value
    for k in reversed(path):
        d = {k: d}
    return d


@pytest.mark.parametrize("seed", range(6))
def test_random_field_values_load_or_raise_config_error(tmp_path, seed):
    import json
    rng = random.Random(seed)
    paths = list(_fields(Config()))
    for i in range(80):
        body = {}
        for _ in range(rng.randint(1, 3)):
            path = rng.choice(paths)
            v = rng.choice(_JUNK)
            if v == ".nan":
                v = float("nan")
            sec = body.setdefault(path[0], {})
            for k in path[1:-1]:
                sec = sec.setdefault(k, {})
            sec[path[-1]] = v
        p = tmp_path / f"c{seed}_{i}.json"
        p.write_text(json.dumps(body))
        try:
            cfg = ConfigLoader(str(p)).load({})
        except ConfigError as e:
            assert str(e)
            continue
        assert isinstance(cfg, Config)


@pytest.mark.parametrize("text,needle", [
    ("engine:\n  max_num_seqs: abc\n", "EngineSection.max_num_seqs"),
    ("model:\n  tensor_parallel_size: [1]\n", "tensor_parallel_size"),
    ("server:\n  port: '80a'\n", "ServerSection.port"),
    ("- a\n- b\n", "mapping"),
    (": :\n", "cannot parse"),
    ("engine:\n  speculative: {num_speculative_tokens: x}\n", "num_speculative_tokens"),
    ("logging: {level: 5}\n", "level"),
    ("server:\n  rate_limit: {enabled: true, requests_per_minute: -5}\n", "requests_per_minute"),
    ("model:\n  max_model_len: 2.5\n", "integer"),
])
def test_malformed_files_name_the_key(tmp_path, text, needle):
    p = tmp_path / "c.yaml"
    p.write_text(text)
    with pytest.raises(ConfigError) as ei:
        ConfigLoader(str(p)).load({})
    assert needle in str(ei.value)


def test_numbers_written_as_strings_are_accepted(tmp_path):
    p = tmp_path / "c.yaml"
    p.write_text("server:\n  port: '9001'\n  api_key: 12345\nengine:\n  gpu_memory_utilization: '0.5'\n"
                 "model:\n  max_model_len: 1e3\n")
    cfg = ConfigLoader(str(p)).load({})
    assert cfg.server.port == 9001 and cfg.server.api_key == "12345"
    assert cfg.engine.gpu_memory_utilization == 0.5 and cfg.model.max_model_len == 1000


@pytest.mark.parametrize("text,needle", [
    ("model:\n  expert_parallel_size: 2\n", "expert_parallel_size"),
    ("model:\n  quantization: {method: fp8_block, group_size: 64}\n", "group_size"),
    ("engine:\n  kv_cache_dtype: int8\n", "kv_cache_dtype"),
    ("engine:\n  scheduling: {enable_preemption: false}\n", "enable_preemption"),
    ("engine:\n  scheduling: {delay_factor: 0.5}\n", "delay_factor"),
])
def test_settings_this_engine_does_not_implement_are_refused(tmp_path, text, needle):
    p = tmp_path / "c.yaml"
    p.write_text(text)
    with pytest.raises(ConfigError) as ei:
        ConfigLoader(str(p)).load({})
    assert needle in str(ei.value)
