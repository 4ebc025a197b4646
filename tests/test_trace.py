"""Host-side trace spans (Chrome trace-event JSON): engine phases recorded through the NVTX
ranges, explicit spans, the event cap, and RUSTEEZE_TRACE writing the file at exit."""
import json
import os
import subprocess
import sys

from rusteeze_b200.metrics import trace

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_engine_phases_and_spans_are_recorded(tmp_path):
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.core.sampling_params import SamplingParams
    from rusteeze_b200.engine.llm_engine import LLMEngine
    path = str(tmp_path / "t.json")
    trace.clear()
    trace.enable(path)
    try:
        cfg = Config()
        cfg.model.device, cfg.model.dtype = "cpu", "float32"
        cfg.engine.num_gpu_blocks = 64
        eng = LLMEngine(cfg)
        with trace.span("test.outer", n=3):
            eng.add_request("r", None, SamplingParams(max_tokens=3, ignore_eos=True), list(range(1, 20)))
            while eng.has_unfinished_requests():
                eng.step()
        assert trace.dump() == path
    finally:
        trace.disable()
    d = json.load(open(path))
    names = {e["name"] for e in d["traceEvents"]}
    assert "rz.step.schedule" in names and "test.outer" in names
    outer = next(e for e in d["traceEvents"] if e["name"] == "test.outer")
    inner = [e for e in d["traceEvents"] if e["name"].startswith("rz.step")]
    assert outer["args"] == {"n": 3} and all(e["ph"] == "X" and e["dur"] >= 0 for e in d["traceEvents"])
    assert all(outer["ts"] <= e["ts"] and e["ts"] + e["dur"] <= outer["ts"] + outer["dur"] + 1 for e in inner)


def test_disabled_tracing_records_nothing_and_the_cap_counts_drops(tmp_path):
    trace.clear()
    with trace.span("x"):
        pass
    assert trace.dump(str(tmp_path / "a.json")) and json.load(open(tmp_path / "a.json"))["traceEvents"] == []
    trace.enable(str(tmp_path / "b.json"), max_events=2)
    try:
        for i in range(5):
            with trace.span(f"s{i}"):
                pass
        trace.dump()
    finally:
        trace.disable()
        trace.clear()
    d = json.load(open(tmp_path / "b.json"))
    assert len(d["traceEvents"]) == 2 and d["otherData"]["dropped_events"] == 3


def test_env_variable_writes_the_trace_at_exit(tmp_path):
    path = tmp_path / "gen.json"
    r = subprocess.run([sys.executable, "-m", "rusteeze_b200", "generate", "-m", "tiny-llama", "--device", "cpu",
                        "--dtype", "float32", "-p", "hi", "--max-tokens", "3"], capture_output=True, text=True,
                       timeout=300, cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT, RUSTEEZE_TRACE=str(path)))
    assert r.returncode == 0, r.stderr
    d = json.load(open(path))
    assert any(e["name"].startswith("rz.step") for e in d["traceEvents"])
