"""`rusteeze benchmark --url`: the HTTP load generator against a real uvicorn server on a
local port (CPU engine, byte-vocabulary model so every step streams a text chunk)."""
import asyncio
import json
import os
import socket
import subprocess
import sys
import threading
import time

import pytest

from rusteeze_b200.api.server import create_app
from rusteeze_b200.config.config import Config
from rusteeze_b200.engine.async_engine import AsyncLLMEngine
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig
from rusteeze_b200.utils.http_bench import run_http_benchmark

BYTES = ModelConfig(name="tiny-bytes", hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                    num_attention_heads=2, num_key_value_heads=1, vocab_size=256, max_position_embeddings=4096)
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def server_url():
    import uvicorn
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device, cfg.model.dtype = "cpu", "float32"
    cfg.engine.num_gpu_blocks, cfg.engine.max_num_seqs, cfg.engine.max_num_batched_tokens = 256, 8, 512
    cfg.engine.enable_chunked_prefill = True
    cfg.logging.request_logging = False
    eng = LLMEngine(cfg, model_config=BYTES)
    step = eng.step
    eng.step = lambda: (time.sleep(0.002), step())[1]      # let the server and clients run
    ae = AsyncLLMEngine(eng).start()
    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    server = uvicorn.Server(uvicorn.Config(create_app(ae, cfg), host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    for _ in range(200):
        if server.started:
            break
        time.sleep(0.05)
    assert server.started
    yield f"http://127.0.0.1:{port}"
    server.should_exit = True
    th.join(timeout=10)
    ae.shutdown()


@pytest.mark.timeout(300)
def test_http_benchmark_counts_every_token(server_url):
    res = asyncio.run(run_http_benchmark(server_url, "tiny-llama", 256, num_prompts=6, input_len=24,
                                         output_len=7, concurrency=3, request_rate=50.0))
    assert res["completed"] == 6 and res["failed"] == 0
    assert res["output_tokens"] == 6 * 7
    assert res["output_tokens_per_s"] > 0 and res["ttft_p50_ms"] > 0 and res["tpot_p50_ms"] > 0
    assert res["ttft_p99_ms"] >= res["ttft_p50_ms"]


@pytest.mark.timeout(300)
def test_cli_benchmark_url(server_url, tmp_path):
    out = tmp_path / "r.json"
    r = subprocess.run([sys.executable, "-m", "rusteeze_b200", "--json", "benchmark", "--url", server_url,
                        "--served-model", "tiny-llama", "--vocab-size", "256", "-n", "4", "--input-len", "16",
                        "--output-len", "5", "--concurrency", "2", "--url-temperature", "0.7", "--url-top-p", "0.9",
                        "-o", str(out)],
                       capture_output=True, text=True, timeout=240, cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0, r.stderr
    d = json.loads(out.read_text())
    assert d["completed"] == 4 and d["output_tokens"] == 20
