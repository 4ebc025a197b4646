"""The OpenAI server over real HTTP (uvicorn on a local port, CPU engine): concurrent
streaming and non-streaming completions, some streams dropped by their clients
mid-generation.  Every kept request completes with its requested length, every dropped
one is aborted in the engine (nothing keeps generating), and the server stays ready."""
import asyncio
import json
import socket
import threading
import time

import pytest

from rusteeze_b200.api.server import create_app
from rusteeze_b200.config.config import Config
from rusteeze_b200.engine.async_engine import AsyncLLMEngine
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig

# a byte-vocabulary model: every sampled token decodes to text, so every step of a stream
# sends a chunk (a 32k-vocabulary random model over the byte tokenizer mostly emits
# tokens without text, and a stream then has nothing to send until it finishes)
BYTES = ModelConfig(name="tiny-bytes", hidden_size=64, intermediate_size=128, num_hidden_layers=1,
                    num_attention_heads=2, num_key_value_heads=1, vocab_size=256, max_position_embeddings=4096)


def _cfg():
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 128
    cfg.engine.max_num_seqs = 8
    cfg.engine.max_num_batched_tokens = 512
    cfg.engine.enable_chunked_prefill = True
    cfg.logging.request_logging = False
    return cfg


@pytest.mark.timeout(300)
def test_concurrent_streams_with_disconnects_over_http():
    import httpx
    import uvicorn
    cfg = _cfg()
    eng = LLMEngine(cfg, model_config=BYTES)
    # the tiny CPU model's step loop holds the GIL almost continuously; a short pause per
    # step lets the server and the clients run, so dropped clients leave mid-generation
    step = eng.step
    eng.step = lambda: (time.sleep(0.005), step())[1]
    ae = AsyncLLMEngine(eng).start()
    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    server = uvicorn.Server(uvicorn.Config(create_app(ae, cfg), host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    base = f"http://127.0.0.1:{port}"
    for _ in range(200):
        if server.started:
            break
        time.sleep(0.05)
    assert server.started

    async def kept(client, i):
        r = await client.post(f"{base}/v1/completions", json={
            "model": "tiny-llama", "prompt": [list(range(65 + i, 85 + i))], "max_tokens": 6 + i % 5,
            "temperature": 0.0})
        assert r.status_code == 200, r.text
        return r.json()["usage"]["completion_tokens"] == 6 + i % 5

    async def kept_stream(client, i):
        text, done = "", False
        async with client.stream("POST", f"{base}/v1/completions", json={
                "model": "tiny-llama", "prompt": [list(range(97 + i, 117 + i))], "max_tokens": 8,
                "temperature": 0.0, "stream": True, "ignore_eos": True}) as r:
            assert r.status_code == 200
            async for line in r.aiter_lines():
                if line == "data: [DONE]":
                    done = True
                elif line.startswith("data: "):
                    text += json.loads(line[6:])["choices"][0]["text"]
        return done

    async def dropped(client, i):
        async with client.stream("POST", f"{base}/v1/completions", json={
                "model": "tiny-llama", "prompt": [list(range(33 + i, 53 + i))], "max_tokens": 5000,
                "temperature": 0.0, "stream": True, "ignore_eos": True}) as r:
            assert r.status_code == 200
            n = 0
            async for line in r.aiter_lines():
                if line.startswith("data: "):
                    n += 1
                    if n == 3:
                        break                     # the client goes away mid-generation
        return True

    async def main():
        async with httpx.AsyncClient(timeout=120) as client:
            res = await asyncio.gather(*([kept(client, i) for i in range(6)] +
                                         [kept_stream(client, i) for i in range(4)] +
                                         [dropped(client, i) for i in range(4)]))
            assert all(res), res
            ready = (await client.get(f"{base}/health/ready")).status_code
            for _ in range(100):                  # the dropped streams are counted once their generators close
                text = (await client.get(f"{base}/metrics")).text
                if 'requests_total{status="aborted"} 4.0' in text:
                    break
                await asyncio.sleep(0.05)
            assert 'requests_total{status="aborted"} 4.0' in text, [ln for ln in text.splitlines()
                                                                     if "requests_total" in ln]
        return ready

    try:
        assert asyncio.run(main()) == 200
        for _ in range(300):                      # the dropped streams are aborted, not left running
            if not eng.has_unfinished_requests():
                break
            time.sleep(0.02)
        assert not eng.has_unfinished_requests(), eng.stats()
        assert eng.stats_counters["requests_aborted"] >= 4
        # kept requests: 6 x (6..10) + 4 x 8 tokens; the dropped streams stop within a few
        # steps of their clients leaving (each could run to 4000 tokens otherwise)
        assert eng.stats_counters["generation_tokens"] < 400
        assert ae.healthy and ae._thread.is_alive()
    finally:
        server.should_exit = True
        th.join(10)
        ae.shutdown()
