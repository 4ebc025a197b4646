"""Load generator for a running OpenAI-compatible server (this engine's or any other):
streamed `/v1/completions` requests of random token ids, sent at a Poisson rate or as fast
as `concurrency` allows, with output tokens counted from the stream's usage chunk.

The reference's `benchmark` command times sleeps (crates/rusteeze-cli/src/commands/
benchmark.rs:97-138); this one measures the public HTTP path end to end: TTFT is the time
to the first streamed token chunk, TPOT the mean gap after it, and output tok/s the
completion tokens of all requests over the wall time from the first send to the last
`[DONE]`.
"""
from __future__ import annotations

import asyncio
import json
import random
import time
from typing import Dict, List, Optional


async def _one(client, url: str, model: str, prompt: List[int], max_tokens: int, sem, out: List[Dict],
               extra: Optional[Dict] = None) -> None:
    body = {"model": model, "prompt": [prompt], "max_tokens": max_tokens, "temperature": 0.0,
            "ignore_eos": True, "stream": True, "stream_options": {"include_usage": True}, **(extra or {})}
    async with sem:
        t0 = time.perf_counter()
        first = last = None
        chunks = 0
        completion = 0
        ok = False
        async with client.stream("POST", url + "/v1/completions", json=body) as r:
            if r.status_code != 200:
                out.append({"ok": False, "status": r.status_code})
                return
            async for line in r.aiter_lines():
                if not line.startswith("data: "):
                    continue
                data = line[6:]
                if data == "[DONE]":
                    ok = True
                    break
                msg = json.loads(data)
                if msg.get("usage"):
                    completion = int(msg["usage"].get("completion_tokens", 0))
                if msg.get("choices") and any(c.get("text") for c in msg["choices"]):
                    now = time.perf_counter()
                    first = first or now
                    last = now
                    chunks += 1
        out.append({"ok": ok, "ttft": None if first is None else first - t0,
                    "tpot": None if chunks < 2 else (last - first) / (chunks - 1),
                    "latency": time.perf_counter() - t0, "completion_tokens": completion})


async def run_http_benchmark(url: str, model: str, vocab: int, num_prompts: int, input_len: int, output_len: int,
                             concurrency: int, request_rate: Optional[float] = None, seed: int = 0,
                             timeout_s: float = 600.0, prompts: Optional[List[List[int]]] = None,
                             output_lens: Optional[List[int]] = None,
                             arrivals: Optional[List[float]] = None, extra_body: Optional[Dict] = None) -> Dict:
    """Random prompts of `input_len` ids and `output_len` tokens each, or an explicit
    workload: `prompts` with their `output_lens`, sent at the `arrivals` offsets (seconds
    from the start) when given."""
    import httpx
    rng = random.Random(seed)
    if prompts is None:
        prompts = [[rng.randrange(vocab) for _ in range(input_len)] for _ in range(num_prompts)]
    olens = output_lens or [output_len] * len(prompts)
    num_prompts = len(prompts)
    sem = asyncio.Semaphore(max(1, concurrency))
    out: List[Dict] = []
    limits = httpx.Limits(max_connections=max(1, concurrency) + 4)
    async with httpx.AsyncClient(timeout=timeout_s, limits=limits) as client:
        t0 = time.perf_counter()
        tasks = []
        for i, p in enumerate(prompts):
            if arrivals is not None:
                await asyncio.sleep(max(0.0, arrivals[i] - (time.perf_counter() - t0)))
            tasks.append(asyncio.create_task(_one(client, url.rstrip("/"), model, p, int(olens[i]), sem, out,
                                                  extra_body)))
            if request_rate and arrivals is None:
                await asyncio.sleep(rng.expovariate(request_rate))
        await asyncio.gather(*tasks)
        wall = time.perf_counter() - t0

    def pct(xs, q):
        xs = sorted(x for x in xs if x is not None)
        if not xs:
            return None
        return xs[min(len(xs) - 1, int(round(q / 100 * (len(xs) - 1))))]

    good = [r for r in out if r["ok"]]
    tokens = sum(r["completion_tokens"] for r in good)
    ms = lambda x: None if x is None else x * 1e3  # noqa: E731
    return {"url": url, "num_prompts": num_prompts, "completed": len(good), "failed": len(out) - len(good),
            "input_len": input_len, "output_len": output_len, "concurrency": concurrency,
            "request_rate": request_rate, "duration_s": wall, "output_tokens": tokens,
            "output_tokens_per_s": tokens / wall if wall > 0 else 0.0,
            "ttft_p50_ms": ms(pct([r["ttft"] for r in good], 50)), "ttft_p99_ms": ms(pct([r["ttft"] for r in good], 99)),
            "tpot_p50_ms": ms(pct([r["tpot"] for r in good], 50)), "tpot_p99_ms": ms(pct([r["tpot"] for r in good], 99)),
            "latency_p50_s": pct([r["latency"] for r in good], 50), "latency_p99_s": pct([r["latency"] for r in good], 99)}
