"""Config precedence (defaults < file < env < CLI), validation, and CLI smoke tests."""
import json
import re
import os
import subprocess
import sys

import pytest

from rusteeze_b200.config.loader import ConfigLoader, env_overrides
from rusteeze_b200.config.validation import collect_errors
from rusteeze_b200.core.errors import ConfigError

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_precedence(tmp_path):
    f = tmp_path / "c.yaml"
    f.write_text("model:\n  preset: tiny-llama\n  dtype: float32\nserver:\n  port: 9000\nengine:\n  max_num_seqs: 32\n")
    env = {"RUSTEEZE_PORT": "9100", "RUSTEEZE_MAX_SEQS": "64"}
    cfg = ConfigLoader(str(f), environ=env).load({"engine": {"max_num_seqs": 128}, "server": {"host": None}})
    assert cfg.model.preset == "tiny-llama"
    assert cfg.server.port == 9100           # env beats file
    assert cfg.engine.max_num_seqs == 128    # CLI beats env
    assert cfg.server.host == "0.0.0.0"      # None CLI values do not override


@pytest.mark.parametrize("ext,text", [
    (".json", '{"engine": {"block_size": 16, "max_num_batched_tokens": 2048}}'),
    (".toml", "[engine]\nblock_size = 16\nmax_num_batched_tokens = 2048\n"),
])
def test_formats(tmp_path, ext, text):
    f = tmp_path / ("c" + ext)
    f.write_text(text)
    cfg = ConfigLoader(str(f), environ={}).load()
    assert cfg.engine.max_num_batched_tokens == 2048


def test_validation_errors(tmp_path):
    f = tmp_path / "bad.yaml"
    f.write_text("model:\n  dtype: int3\n  device: metal\n  pipeline_parallel_size: 2\nengine:\n  block_size: 32\n")
    cfg = ConfigLoader(str(f), environ={}).load(validate=False)
    errs = collect_errors(cfg)
    assert any("dtype" in e for e in errs) and any("device" in e for e in errs)
    assert any("pipeline_parallel_size" in e for e in errs) and any("block_size" in e for e in errs)
    with pytest.raises(ConfigError):
        ConfigLoader(str(f), environ={}).load()


def test_unknown_key_rejected(tmp_path):
    f = tmp_path / "u.yaml"
    f.write_text("engine:\n  no_such_knob: 1\n")
    with pytest.raises(ConfigError):
        ConfigLoader(str(f), environ={}).load()


def test_env_override_types():
    assert env_overrides(environ={"RUSTEEZE_GPU_MEMORY_UTIL": "0.5"})["engine"]["gpu_memory_utilization"] == 0.5
    with pytest.raises(ConfigError):
        env_overrides(environ={"RUSTEEZE_PORT": "abc"})


def test_example_config_is_valid():
    cfg = ConfigLoader(os.path.join(ROOT, "config.example.yaml"), environ={}).load()
    assert cfg.engine.block_size == 16


def _cli(*args, stdin=None):
    env = dict(os.environ, PYTHONPATH=ROOT)
    return subprocess.run([sys.executable, "-m", "rusteeze_b200", *args], capture_output=True, text=True,
                          cwd=ROOT, env=env, input=stdin, timeout=300)


def test_cli_version_info_validate(tmp_path):
    r = _cli("--json", "version")
    assert r.returncode == 0 and json.loads(r.stdout)["version"]
    r = _cli("info", "llama-3-8b")
    d = json.loads(r.stdout)
    assert 7.9 < d["parameters_billions"] < 8.1
    f = tmp_path / "c.yaml"
    f.write_text("engine:\n  block_size: 32\n")
    r = _cli("--json", "validate", str(f))
    assert r.returncode == 1 and not json.loads(r.stdout)["valid"]


def test_cli_generate_and_benchmark_tiny():
    r = _cli("--json", "generate", "-m", "tiny-llama", "--device", "cpu", "--dtype", "float32", "-p", "hello",
             "--max-tokens", "4", "--temperature", "0")
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert len(out[0]["outputs"][0]["token_ids"]) == 4
    r = _cli("--json", "benchmark", "-m", "tiny-llama", "--device", "cpu", "--dtype", "float32", "-n", "4",
             "--input-len", "16", "--output-len", "4", "--concurrency", "4", "--warmup", "1")
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout)["output_tokens_per_s"] > 0


def test_cli_generate_beam_search_and_structured_output(tmp_path):
    base = ("--json", "generate", "-m", "tiny-llama", "--device", "cpu", "--dtype", "float32", "-p", "hello")
    r = _cli(*base, "--max-tokens", "20", "--regex", "[0-9]{3}-[a-z]{2}")
    assert r.returncode == 0, r.stderr
    assert re.fullmatch("[0-9]{3}-[a-z]{2}", json.loads(r.stdout)[0]["outputs"][0]["text"])
    r = _cli(*base, "--max-tokens", "10", "--choice", "red", "--choice", "blue", "-n", "2")
    assert {c["text"] for c in json.loads(r.stdout)[0]["outputs"]} <= {"red", "blue"}
    schema = tmp_path / "s.json"
    schema.write_text(json.dumps({"type": "object", "properties": {"ok": {"type": "boolean"}}, "required": ["ok"]}))
    r = _cli(*base, "--max-tokens", "40", "--json-schema", str(schema), "--temperature", "0")
    assert r.returncode == 0, r.stderr
    assert isinstance(json.loads(json.loads(r.stdout)[0]["outputs"][0]["text"])["ok"], bool)
    r = _cli(*base, "--max-tokens", "4", "--beam-width", "3", "-n", "2")
    assert r.returncode == 0, r.stderr
    assert len(json.loads(r.stdout)[0]["outputs"]) == 2


def test_cli_rejects_pipeline_parallel():
    r = _cli("serve", "-m", "tiny-llama", "--pipeline-parallel-size", "2")
    assert r.returncode == 2 and "pipeline_parallel_size" in r.stderr


def test_serve_options_not_given_keep_the_config_file_values(tmp_path, monkeypatch):
    """`rusteeze -c file serve` with no flags: the file's values stand (argparse defaults used
    to override them); flags given on the command line still win."""
    from rusteeze_b200.cli.main import _load_config, build_parser
    p = tmp_path / "c.yaml"
    p.write_text("model:\n  preset: tiny-llama\n  tensor_parallel_size: 2\n  dtype: float32\n"
                 "engine:\n  max_num_seqs: 96\n  max_num_batched_tokens: 2048\n  swap_space_gb: 1.5\n"
                 "server:\n  port: 9001\n  router_policy: round_robin\n")
    for k in ("RUSTEEZE_MODEL", "RUSTEEZE_PORT", "RUSTEEZE_MAX_SEQS", "RUSTEEZE_CONFIG"):
        monkeypatch.delenv(k, raising=False)
    a = build_parser().parse_args(["-c", str(p), "serve"])
    cfg = _load_config(a, {"server": {"port": a.port}, "engine": {"max_num_seqs": a.max_num_seqs,
                                                                   "swap_space_gb": a.swap_space}})
    assert (cfg.model.tensor_parallel_size, cfg.model.dtype, cfg.engine.max_num_seqs) == (2, "float32", 96)
    assert (cfg.engine.max_num_batched_tokens, cfg.engine.swap_space_gb, cfg.server.port) == (2048, 1.5, 9001)
    assert cfg.server.router_policy == "round_robin"
    a = build_parser().parse_args(["-c", str(p), "serve", "--max-num-seqs", "8", "-p", "9100"])
    cfg = _load_config(a, {"server": {"port": a.port}, "engine": {"max_num_seqs": a.max_num_seqs}})
    assert (cfg.engine.max_num_seqs, cfg.server.port, cfg.model.tensor_parallel_size) == (8, 9100, 2)


def test_a_model_is_required_from_somewhere(tmp_path, monkeypatch):
    import pytest
    from rusteeze_b200.cli.main import _load_config, build_parser
    for k in ("RUSTEEZE_MODEL", "RUSTEEZE_CONFIG", "RUSTEEZE_MODEL_PATH", "RUSTEEZE_MODEL_PRESET"):
        monkeypatch.delenv(k, raising=False)
    with pytest.raises(SystemExit):
        _load_config(build_parser().parse_args(["serve"]))
    monkeypatch.setenv("RUSTEEZE_MODEL", "tiny-llama")
    assert _load_config(build_parser().parse_args(["serve"])).model.preset == "tiny-llama"


def test_validate_accepts_the_newer_knobs_and_refuses_bad_values(tmp_path):
    good = tmp_path / "good.yaml"
    good.write_text("engine:\n  speculative: {method: ngram, num_speculative_tokens: 4, ngram_max: 4, ngram_min: 1}\n"
                    "metrics:\n  push_gateway: {url: 'http://gw:9091', job: rz}\n"
                    "server:\n  router_policy: prefix_affinity\n"
                    "  rate_limit: {enabled: true, tokens_per_minute: 1000, tokens_per_day: 100000}\n")
    r = _cli("-c", str(good), "validate")
    assert r.returncode == 0 and "valid" in r.stdout, r.stderr
    bad = tmp_path / "bad.yaml"
    bad.write_text("engine:\n  speculative: {method: medusa}\nmetrics:\n  push_gateway: {url: 'gw', job: ''}\n"
                   "server:\n  router_policy: sticky\n  rate_limit: {enabled: true, tokens_per_minute: 0}\n")
    r = _cli("-c", str(bad), "validate")
    assert r.returncode != 0
    for needle in ("medusa", "push_gateway.url", "push_gateway.job", "router_policy", "tokens_per_minute"):
        assert needle in r.stdout + r.stderr, needle
