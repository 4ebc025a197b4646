#!/usr/bin/env python
"""Serving benchmark: output tokens/s of continuous-batched Llama-3-8B.

Workload (synthetic requests, random-init N(0, 0.02) weights of the named
architecture; no network for checkpoints or datasets):
  * Llama-3-8B: 32 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128,
    intermediate 14336, vocab 128256, RoPE theta 5e5; block-scaled fp8 e4m3
    weights (128x128 weight scales, 1x128 activation scales, both powers of
    two so the tensor core applies them: MXFP8 / UE8M0), bf16 activations
    and KV (`--dtype bf16` runs unquantised bf16 weights).
  * Requests with prompt lengths uniform in [128, 2048], output lengths
    uniform in [64, 512], top-p 0.9 at temperature 0.7, Poisson arrivals
    (1024 requests per GPU), served with continuous batching, paged KV
    (block 16), chunked prefill, max 256 running sequences.

N GPUs (torchrun, one rank per GPU) run ONE tensor-parallel engine over all of
them (`--parallel tp`, the default at N > 1): rank 0 schedules and samples,
every rank runs the forward on its weight shard, and the layer boundaries are
the fused GEMM + reduce-scatter / add + RMSNorm + all-gather kernels over
NVLink (`--comm fused`; `--comm nccl` is the NCCL baseline).  Scaling is weak
by default: the engine serves N x 1024 requests at N x the arrival rate with
N x 256 running sequences and N x the prefill budget, so every GPU carries the
1-GPU run's per-GPU load (`--scaling strong` keeps the 1-GPU workload).
`--parallel dp` runs one independent replica per GPU instead.
  1. ramp: engine steps until the running batch is full and half a batch of
     requests has finished (untimed)
  2. W warm-up engine steps (untimed)
  3. K timed engine steps, bracketed by a barrier + cuda synchronize and
     timed with CUDA events on the engine's stream on every rank; MAX over ranks.
  value = output tokens produced in the K steps / max time over ranks.
  e2e: a separate run through the public `LLMEngine` API (add_request /
     step) that serves a fresh request stream of the same shape (same count,
     lengths and Poisson arrival rate; each request is submitted when its
     arrival time has passed) from the first submission to the last token;
     every step copies its inputs from pinned host memory and reads the
     sampled tokens back.
The inputs (weights + KV working set) are far larger than the 126 MB L2, so
no L2 flush is needed between steps.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
Multi-GPU: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REFERENCE_PUBLISHED_TOK_S = 32000.0   # the reference README's output tok/s at batch 256 (A100, Llama-2-7B)
REFERENCE_PUBLISHED_BASIS = ("reference README claim: 32,000 output tok/s, Llama-2-7B static batch 256 on one "
                             "A100 80GB (README.md:88); a different model, workload and GPU, and not reproducible "
                             "by the reference's own code")


def reference_unavailable() -> str:
    return ("reference is a Rust/cargo workspace (no setup.py/pyproject, pip install --target fails: "
            "'not installable'); no cargo/rustc in this image, and its engine samples from all-zero "
            "logits without calling a model (crates/rusteeze-engine/src/engine.rs:418-427)")


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        return summarize_clocks(self.lines)


class Device:
    """The measured device: CUDA events and synchronisation on a GPU; the host clock on
    CPU, where tiny models exercise the harness itself (those runs are not benchmarks)."""

    def __init__(self, device: str):
        import torch
        self.torch = torch
        self.name = device
        self.cuda = device.startswith("cuda")

    def sync(self) -> None:
        if self.cuda:
            self.torch.cuda.synchronize()

    def stream(self):
        return self.torch.cuda.current_stream() if self.cuda else None

    def event(self) -> "Event":
        return Event(self)

    def nvtx(self, name: str = None) -> None:
        if self.cuda:
            if name is None:
                self.torch.cuda.nvtx.range_pop()
            else:
                self.torch.cuda.nvtx.range_push(name)

    def kernel_status(self) -> int:
        if not self.cuda:
            return 0
        from rusteeze_b200 import ops
        return int(ops.cuda_ext().status()[0])

    def pinned(self, values):
        t = self.torch.tensor(values, dtype=self.torch.int64)
        return t.pin_memory() if self.cuda else t


class Event:
    def __init__(self, dev: Device):
        self.dev = dev
        self.ev = dev.torch.cuda.Event(enable_timing=True) if dev.cuda else None
        self.t = None

    def record(self, stream=None) -> None:
        if self.ev is not None:
            self.ev.record(stream) if stream is not None else self.ev.record()
        else:
            self.t = time.perf_counter()

    def elapsed_ms(self, end: "Event") -> float:
        return self.ev.elapsed_time(end.ev) if self.ev is not None else (end.t - self.t) * 1e3


def summarize_clocks(lines) -> dict:
    """nvidia-smi samples (clocks.sm, clocks.max.sm, power, active mask, then the four
    throttle reasons as Active / Not Active) -> median SM clock, max clock and every
    throttle reason seen active."""
    sm, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for ln in lines:
        parts = [p.strip() for p in ln.split(",")]
        if len(parts) < 8:
            continue
        try:
            sm.append(float(parts[0]))
            mx = float(parts[1])
        except ValueError:
            continue
        for n, v in zip(names, parts[4:8]):
            if v.lower().startswith("active"):
                reasons.add(n)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
            "reasons": sorted(reasons), "samples": len(sm)}


def build_workload(n, seed, vocab, rate, prompt_len=(128, 2048), output_len=(64, 512)):
    import numpy as np
    rng = np.random.default_rng(seed)
    plen = rng.integers(prompt_len[0], prompt_len[1] + 1, n)
    olen = rng.integers(output_len[0], output_len[1] + 1, n)
    gaps = rng.exponential(1.0 / rate, n)
    arrivals = np.cumsum(gaps)
    prompts = [rng.integers(0, vocab, int(p)).tolist() for p in plen]
    return prompts, olen.tolist(), arrivals.tolist()


def make_engine(args, device):
    from rusteeze_b200.engine.llm_engine import LLMEngine
    return LLMEngine(make_config(args, device))


def make_config(args, device):
    from rusteeze_b200.config.config import Config
    cfg = Config()
    cfg.model.preset = args.model
    cfg.model.device = device
    cfg.model.dtype = "bfloat16" if device.startswith("cuda") else "float32"
    cfg.model.seed = 0
    if not device.startswith("cuda"):
        cfg.engine.num_gpu_blocks = 512          # host-memory KV for the tiny harness models
    if args.dtype == "fp8":
        from rusteeze_b200.config.config import QuantizationConfig
        cfg.model.quantization = QuantizationConfig(method="fp8_block")
    cfg.engine.max_num_seqs = args.max_seqs
    cfg.engine.max_num_batched_tokens = args.max_batched_tokens
    cfg.engine.kv_cache_dtype = getattr(args, "kv_cache_dtype", "auto")
    cfg.engine.enable_chunked_prefill = True
    cfg.engine.gpu_memory_utilization = 0.88
    cfg.engine.swap_space_gb = 0
    cfg.engine.cuda_graph_max_batch = args.max_seqs
    cfg.engine.enforce_eager = bool(getattr(args, "eager", False))
    if args.workload == "shared-prefix":
        cfg.engine.enable_prefix_caching = True
    if args.draft:
        from rusteeze_b200.config.config import SpeculativeSection
        if args.draft == "ngram":
            cfg.engine.speculative = SpeculativeSection(method="ngram", num_speculative_tokens=args.spec_k)
        else:
            cfg.engine.speculative = SpeculativeSection(
                draft_preset=None if args.draft == "self" else args.draft, num_speculative_tokens=args.spec_k)
        # a verify pass holds max_num_seqs * (k + 1) tokens
        cfg.engine.max_num_batched_tokens = max(cfg.engine.max_num_batched_tokens,
                                                args.max_seqs * (args.spec_k + 1))
    return cfg


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="rusteeze", choices=["rusteeze", "reference"])
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--requests", type=int, default=1024)
    ap.add_argument("--rate", type=float, default=200.0, help="Poisson arrival rate per GPU (req/s)")
    ap.add_argument("--max-seqs", type=int, default=256)
    ap.add_argument("--max-batched-tokens", type=int, default=4096)
    ap.add_argument("--e2e-requests", type=int, default=None,
                    help="requests of the end-to-end run (default: --requests, scaled like it)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-http", action="store_true",
                    help="run the end-to-end stream through the HTTP server (streamed /v1/completions calls) "
                         "instead of LLMEngine.add_request (one engine, one process)")
    ap.add_argument("--dtype", default="fp8", choices=["fp8", "bf16"],
                    help="fp8: block-scaled e4m3 weights (the Llama-3-8B serving configuration); bf16: unquantised")
    ap.add_argument("--fp8", action="store_true", help="same as --dtype fp8 (the default)")
    ap.add_argument("--kv-cache-dtype", default="auto", choices=["auto", "fp8_e4m3", "fp8_e5m2"],
                    help="paged KV cache element type (auto: bf16, the configuration the headline is quoted on)")
    ap.add_argument("--eager", action="store_true", help="disable CUDA graphs (profiling runs)")
    ap.add_argument("--parallel", default=None, choices=["dp", "tp"],
                    help="tp: one tensor-parallel engine over all GPUs (default with N > 1); dp: one engine "
                         "replica per GPU")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="tp: weak = requests, arrival rate, running sequences and prefill budget x N "
                         "(per-GPU load of the 1-GPU run); strong = the 1-GPU workload on N GPUs")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                    help="tensor-parallel collectives: fused peer-memory kernels or the NCCL baseline")
    ap.add_argument("--workload", default="poisson", choices=["poisson", "static", "shared-prefix"],
                    help="poisson: continuous batching (default); static: batches of --batches requests, "
                         "--static-prompt prompt tokens, --static-output greedy tokens (README table shape); "
                         "shared-prefix: static batches whose prompts share a --shared-prefix token prefix "
                         "followed by --static-prompt unique tokens (prefix caching on)")
    ap.add_argument("--shared-prefix", type=int, default=1024)
    ap.add_argument("--draft", default=None,
                    help="speculative decoding: random-init draft preset (e.g. llama-3.2-1b), 'self', or 'ngram' "
                         "(prompt lookup, no draft model)")
    ap.add_argument("--spec-k", type=int, default=4, help="draft tokens per speculative round")
    ap.add_argument("--batches", default="1,8,32,128,256")
    ap.add_argument("--device", default="cuda", choices=["cuda", "cpu"],
                    help="cpu runs the harness itself on tiny models (gloo ranks, host clock): not a benchmark")
    ap.add_argument("--prompt-len", default="128,2048", help="prompt length range of the Poisson workload")
    ap.add_argument("--output-len", default="64,512", help="output length range of the Poisson workload")
    ap.add_argument("--op-split", type=int, default=0,
                    help="after the timed window, run this many more steps with per-section CUDA events "
                         "(GEMMs with their collectives, attention, norms, sampling; MAX over ranks) and "
                         "report ms per step per section; not part of the timed value")
    ap.add_argument("--static-prompt", type=int, default=512)
    ap.add_argument("--static-output", type=int, default=128)
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reference_unavailable(),
                              "metric": "output_tokens_per_s", "n_gpus": args.gpus}))
        return 0

    import torch
    import torch.distributed as dist

    cuda = args.device == "cuda"
    if cuda:
        torch.cuda.set_device(local)
    if args.parallel is None:
        args.parallel = "tp" if world > 1 else "dp"
    if args.e2e_requests is None:
        args.e2e_requests = args.requests
    if world > 1 and args.parallel == "tp":
        return serve_tp(args, world, rank)
    if world > 1:
        from datetime import timedelta
        if cuda:
            dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    device = f"cuda:{local}" if cuda else "cpu"
    eng = make_engine(args, device)
    if args.workload != "poisson":
        static_batches(args, eng, device, rank, world)
    else:
        line = serve(args, eng, device, rank, local, world)
        if rank == 0:
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def serve_tp(args, world, rank):
    """Tensor-parallel serving of the same workload: ONE engine over all N GPUs.
    Rank 0 schedules and samples; ranks 1..N-1 run the forward on their weight
    shard from the plan ring; the collectives are the fused peer-memory kernels
    (`--comm fused`: GEMM + reduce-scatter, add + RMSNorm + all-gather) or NCCL.
    Timed windows come from `TPExecutor.timer` (CUDA events on every rank, MAX)."""
    import torch
    import torch.distributed as dist
    from rusteeze_b200.parallel.dist import init_distributed
    from rusteeze_b200.parallel.executor import worker_loop
    from rusteeze_b200.parallel.launcher import tp_rank_setup
    info = init_distributed(timeout_s=600, device_type=args.device)
    if args.scaling == "weak":
        # every GPU carries the 1-GPU run's load: N x the requests, arrival rate, running
        # sequences and prefill budget on the one N-GPU engine
        args.requests *= world
        args.e2e_requests *= world
        args.rate *= world
        args.max_seqs *= world
        args.max_batched_tokens *= world
    cfg = make_config(args, str(info.device))
    cfg.model.tensor_parallel_size = world
    cfg.engine.comm_backend = args.comm
    eng, runner, channel = tp_rank_setup(cfg, info, tag=f"bench{os.environ.get('MASTER_PORT', '0')}")
    try:
        if rank != 0:
            worker_loop(runner, channel)
            return 0
        try:
            if args.workload != "poisson":
                static_batches(args, eng, str(info.device), 0, 1, tp_timer=eng.runner.timer)
                return 0
            line = serve(args, eng, str(info.device), 0, int(os.environ.get("LOCAL_RANK", "0")), 1,
                         tp_timer=eng.runner.timer)
        finally:
            eng.runner.shutdown()
        line.update(n_gpus=world, scaling=args.scaling, gpu_launches_scope="rank 0")
        line["config"]["parallelism"] = f"tp{world} ({args.comm} collectives)"
        line["config"]["global_batch"] = args.max_seqs
        line["config"]["workload"] = line["config"]["workload"].replace("req/GPU", "req").replace(
            "/s,", "/s in total,")
        print(json.dumps(line), flush=True)
        return 0
    finally:
        runner.release_graphs()            # graphs holding NCCL calls go before the process group
        Device(str(info.device)).sync()
        dist.destroy_process_group()


def e2e_over_http(eng, V, prompts, olens, arrivals, dev):
    """The end-to-end run through the OpenAI-compatible HTTP server (one process, one
    engine): the server runs in this process on a local port, and every request of the
    stream is a streamed /v1/completions call sent at its Poisson arrival time; output
    tok/s over the wall time from the first send to the last [DONE]."""
    import asyncio
    import socket
    import threading
    import uvicorn
    from rusteeze_b200.api.server import create_app
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.engine.async_engine import AsyncLLMEngine
    from rusteeze_b200.utils.http_bench import run_http_benchmark
    cfg = Config()
    cfg.logging.request_logging = False
    cfg.server.max_connections = max(cfg.server.max_connections, len(prompts) + 16)
    h2d0, d2h0, steps0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes, eng.stats_counters["steps"]
    ae = AsyncLLMEngine(eng).start()
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    port = sk.getsockname()[1]
    sk.close()
    server = uvicorn.Server(uvicorn.Config(create_app(ae, cfg), host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    t_wait = time.monotonic()
    while not server.started and time.monotonic() - t_wait < 60:
        time.sleep(0.05)
    try:
        res = asyncio.run(run_http_benchmark(
            f"http://127.0.0.1:{port}", "", V, len(prompts), 0, 0, concurrency=len(prompts),
            prompts=[list(map(int, p)) for p in prompts], output_lens=[int(x) for x in olens],
            arrivals=[float(a) for a in arrivals], extra_body={"temperature": 0.7, "top_p": 0.9}))
    finally:
        server.should_exit = True
        th.join(30)
        ae.shutdown()
    dev.sync()
    steps = max(1, eng.stats_counters["steps"] - steps0)
    return {"value": res["output_tokens_per_s"], "unit": "output_tokens/s",
            "h2d_bytes_per_step": int((eng.runner.h2d_bytes - h2d0) / steps),
            "d2h_bytes_per_step": int((eng.runner.d2h_bytes - d2h0) / steps),
            "requests": res["num_prompts"], "completed": res["completed"], "wall_s": round(res["duration_s"], 3),
            "via": "http",
            "workload": f"{len(prompts)} requests, Poisson {len(prompts) / max(arrivals[-1], 1e-9):.0f}/s arrivals, "
                        "same length ranges and sampling as the timed run, each a streamed /v1/completions call "
                        "to the in-process HTTP server; wall clock from the first send to the last [DONE]",
            "ttft_p50_s": None if res["ttft_p50_ms"] is None else round(res["ttft_p50_ms"] / 1e3, 4)}


def serve(args, eng, device, rank, local, world, tp_timer=None):
    """The serving measurement on one engine: ramp to steady state, W warm-up
    steps, K device-timed steps, then the end-to-end run through the public API.
    `world` > 1 means data-parallel replicas (every rank runs this; MAX / SUM over
    ranks); with `tp_timer` (tensor parallel) only rank 0 runs it and the timer
    takes the MAX over the TP ranks.  Returns the JSON line (rank 0)."""
    import torch
    import torch.distributed as dist
    from rusteeze_b200 import ops
    from rusteeze_b200.core.sampling_params import SamplingParams
    dev = Device(device)
    V = eng.model_config.vocab_size
    plen = tuple(int(x) for x in args.prompt_len.split(","))
    olen = tuple(int(x) for x in args.output_len.split(","))
    prompts, olens, arrivals = build_workload(args.requests, 1000, V, args.rate, plen, olen)
    eng_stream = dev.stream()

    # ---------------------------------------------------------------- steady-state serving
    t0 = time.monotonic()
    nxt = 0
    req_ids = {}

    def admit(now):
        nonlocal nxt
        while nxt < len(prompts) and arrivals[nxt] <= now:
            sp = SamplingParams(temperature=0.7, top_p=0.9, max_tokens=int(olens[nxt]), ignore_eos=True,
                                output_kind="final_only")
            r = eng.add_request(None, None, sp, prompts[nxt])
            req_ids[r.request_id] = nxt
            nxt += 1

    def step():
        now = time.monotonic() - t0
        admit(now)
        if not eng.has_unfinished_requests() and nxt < len(prompts):
            time.sleep(max(0.0, min(0.05, arrivals[nxt] - now)))   # idle until the next arrival
            admit(time.monotonic() - t0)
        return eng.step()

    # 1. ramp to steady state (bounded by wall time): the batch is full AND half
    #    a batch of requests has already finished, so the timed steps mix decode
    #    with the prefill of newly admitted requests instead of measuring the
    #    decode-only phase right after the first admissions
    ramp_steps = 0
    ramp_deadline = time.monotonic() + 300.0
    finished0 = eng.stats_counters["requests_finished"]
    while time.monotonic() < ramp_deadline:
        if (eng.scheduler.num_running >= args.max_seqs and
                eng.stats_counters["requests_finished"] - finished0 >= args.max_seqs // 2):
            break
        step()
        ramp_steps += 1
        if nxt >= len(prompts) and not eng.has_unfinished_requests():
            break
    # 2. warm-up
    for _ in range(args.warmup):
        step()
    # 3. timed
    gen0 = eng.stats_counters["generation_tokens"]
    prompt0 = eng.stats_counters["prompt_tokens"]
    phase0 = eng.host_phase_seconds()
    launches0 = ops.launch_count()
    if world > 1:
        dist.barrier()
    dev.sync()
    clk = ClockSampler(local)
    clk.start()
    ev0, ev1 = dev.event(), dev.event()
    if tp_timer is not None:
        tp_timer("start")
    ev0.record(eng_stream)
    ttfts, tpots = [], []
    dev.nvtx("rz_timed")       # lets ncu --nvtx-include select steady-state launches
    for _ in range(args.steps):
        for out in step():
            if out.finished and out.metrics is not None:
                if out.metrics.ttft is not None:
                    ttfts.append(out.metrics.ttft)
                if out.metrics.tpot is not None:
                    tpots.append(out.metrics.tpot)
    dev.nvtx()
    ev1.record(eng_stream)
    tp_ms = tp_timer("stop") if tp_timer is not None else None
    dev.sync()
    if world > 1:
        dist.barrier()
    clocks = clk.stop()
    ms = ev0.elapsed_ms(ev1) if tp_ms is None else tp_ms
    launches = ops.launch_count() - launches0
    gen = eng.stats_counters["generation_tokens"] - gen0
    prompt_toks = eng.stats_counters["prompt_tokens"] - prompt0
    phase1 = eng.host_phase_seconds()
    host_ms = {k: round((phase1[k] - phase0.get(k, 0.0)) * 1e3 / max(1, args.steps), 3) for k in phase1}
    status = dev.kernel_status()

    t = torch.tensor([ms, float(gen), float(launches)], dtype=torch.float64, device=device)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        ms_max, gen_sum, launches_sum = tmax[0].item(), tsum[1].item(), tsum[2].item()
    else:
        ms_max, gen_sum, launches_sum = ms, float(gen), float(launches)
    value = gen_sum / (ms_max / 1000.0)

    # ---------------------------------------------------------------- per-section split (separate window)
    op_split = None
    if args.op_split > 0 and dev.cuda:
        from rusteeze_b200.utils.op_timer import OP_TIMER, SECTIONS
        if tp_timer is not None:
            tp_timer("ops_start")
        else:
            OP_TIMER.start()
        sg0 = eng.stats_counters["steps"]
        for _ in range(args.op_split):
            step()
        dev.sync()
        if tp_timer is not None:
            rep = tp_timer("ops_stop")
        else:
            OP_TIMER.stop()
            rep = OP_TIMER.report()
            if world > 1:
                tv = torch.tensor([rep.get(k, 0.0) for k in SECTIONS], dtype=torch.float64, device=device)
                dist.all_reduce(tv, op=dist.ReduceOp.MAX)
                rep = dict(zip(SECTIONS, tv.tolist()))
        n_st = max(1, eng.stats_counters["steps"] - sg0)
        op_split = {"steps": n_st, "ms_per_step": {k: round(v / n_st, 3) for k, v in rep.items() if v > 0},
                    "note": "CUDA events around each section on the engine stream, MAX over ranks; the "
                            "events break the overlap between fused sections, so the sum exceeds ms_per_step"}

    # ---------------------------------------------------------------- end-to-end through the public API
    e2e = None
    http_e2e = bool(getattr(args, "e2e_http", False)) and world == 1 and tp_timer is None
    if not args.no_e2e and http_e2e:
        for rid in list(eng.requests):
            eng.abort_request(rid)
        e_prompts, e_olens, e_arr = build_workload(args.e2e_requests, 5000, V, args.rate, plen, olen)
        e2e = e2e_over_http(eng, V, e_prompts, e_olens, e_arr, dev)
    if not args.no_e2e and not http_e2e:
        # drain the steady-state run so the e2e run starts from an empty engine
        for rid in list(eng.requests):
            eng.abort_request(rid)
        e_prompts, e_olens, e_arr = build_workload(args.e2e_requests, 5000, V, args.rate, plen, olen)
        h2d0, d2h0, steps0 = eng.runner.h2d_bytes, eng.runner.d2h_bytes, eng.stats_counters["steps"]
        gen_e0 = eng.stats_counters["generation_tokens"]
        if world > 1:
            dist.barrier()
        dev.sync()
        w0 = time.perf_counter()
        e_next = 0
        e_ttft = []
        while e_next < len(e_prompts) or eng.has_unfinished_requests():
            now = time.perf_counter() - w0
            while e_next < len(e_prompts) and e_arr[e_next] <= now:   # Poisson arrivals, as in config 3
                eng.add_request(None, None, SamplingParams(temperature=0.7, top_p=0.9,
                                                           max_tokens=int(e_olens[e_next]), ignore_eos=True,
                                                           output_kind="final_only"),
                                e_prompts[e_next])
                e_next += 1
            if not eng.has_unfinished_requests():
                time.sleep(max(0.0, min(0.05, e_arr[e_next] - now)))
                continue
            for out in eng.step():
                if out.finished and out.metrics is not None and out.metrics.ttft is not None:
                    e_ttft.append(out.metrics.ttft)
        dev.sync()
        w1 = time.perf_counter()
        if world > 1:
            dist.barrier()
        egen = eng.stats_counters["generation_tokens"] - gen_e0
        esteps = max(1, eng.stats_counters["steps"] - steps0)
        et = torch.tensor([w1 - w0, float(egen)], dtype=torch.float64, device=device)
        if world > 1:
            emax = et.clone()
            dist.all_reduce(emax, op=dist.ReduceOp.MAX)
            esum = et.clone()
            dist.all_reduce(esum, op=dist.ReduceOp.SUM)
            e_s, e_gen = emax[0].item(), esum[1].item()
        else:
            e_s, e_gen = et[0].item(), et[1].item()
        e2e = {"value": e_gen / e_s, "unit": "output_tokens/s",
               "h2d_bytes_per_step": int((eng.runner.h2d_bytes - h2d0) / esteps),
               "d2h_bytes_per_step": int((eng.runner.d2h_bytes - d2h0) / esteps),
               "requests": args.e2e_requests * world, "wall_s": round(e_s, 3),
               "workload": f"{args.e2e_requests} requests per engine, Poisson {args.rate}/s arrivals, same "
                           "length ranges and sampling as the timed run, submitted through LLMEngine.add_request "
                           "as they arrive (output_kind final_only: one output with its detokenised text per "
                           "request); wall clock from the first submission to the last token",
               "ttft_p50_s": round(statistics.median(e_ttft), 4) if e_ttft else None}

    line = {
        "metric": "output_tokens_per_s",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(value / REFERENCE_PUBLISHED_TOK_S, 4),
        "vs_baseline_basis": REFERENCE_PUBLISHED_BASIS,
        "dtype": (("fp8_e4m3 weights (128x128 UE8M0 block scales), 1x128 UE8M0 activation scales, "
                   "bf16 activations, fp32 accumulate") if args.dtype == "fp8" else "bf16")
                 + (", bf16 KV cache" if args.kv_cache_dtype == "auto" else f", {args.kv_cache_dtype} KV cache"),
        "data": "synthetic requests, random-init N(0,0.02) weights",
        "config": {"model": args.model, "global_batch": args.max_seqs * world,
                   "seq_len": "prompt U[{},{}] + output U[{},{}]".format(*plen, *olen),
                   "parallelism": f"dp{world}" if world > 1 else "tp1",
                   "workload": f"{args.requests} req/GPU Poisson {args.rate}/s, top_p 0.9 T 0.7, "
                               "continuous batching, paged KV block 16, chunked prefill "
                               f"{args.max_batched_tokens} tok/step",
                   "l2": "working set (16 GB weights + KV) far exceeds the 126 MB L2; no flush",
                   "ramp_steps": ramp_steps},
        "ttft_p50_s": round(statistics.median(ttfts), 4) if ttfts else None,
        "tpot_p50_s": round(statistics.median(tpots), 5) if tpots else None,
        "prompt_tokens_per_step": round(prompt_toks / max(1, args.steps), 1),
        "host_ms_per_step": host_ms,
        "clocks": clocks,
        "gpu_launches": int(launches_sum),
        "kernel_status": status,
        "e2e": e2e,
    }
    if op_split is not None:
        line["op_split"] = op_split
    return line


def static_batches(args, eng, device, rank, world, tp_timer=None):
    """Static batches (all requests admitted together, greedy, EOS ignored):
    for each batch size B, B prompts decode --static-output tokens; output
    tok/s = B * output / (device time from the first step to the last token),
    timed with CUDA events, MAX over ranks (DP replicas: `world` > 1; one
    tensor-parallel engine: `tp_timer`).  Prompts are --static-prompt random
    tokens, or with `--workload shared-prefix` a common --shared-prefix-token
    random prefix plus a unique --static-prompt-token suffix (prefix caching on).
    One JSON line per batch size."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from rusteeze_b200.core.sampling_params import SamplingParams
    dev = Device(device)
    V = eng.model_config.vocab_size
    rng = np.random.default_rng(0)
    prefix = rng.integers(0, V, args.shared_prefix).tolist() if args.workload == "shared-prefix" else []
    stream = dev.stream()
    for B in [int(x) for x in args.batches.split(",")]:
        def run_once():
            for _ in range(B):
                eng.add_request(None, None, SamplingParams(temperature=0.0, max_tokens=args.static_output,
                                                           ignore_eos=True, output_kind="final_only"),
                                prefix + rng.integers(0, V, args.static_prompt).tolist())
            ttft = []
            while eng.has_unfinished_requests():
                for o in eng.step():
                    if o.finished and o.metrics.ttft is not None:
                        ttft.append(o.metrics.ttft)
            return ttft
        run_once()                                   # warm-up (graphs, allocator, prefix cache)
        if world > 1:
            dist.barrier()
        dev.sync()
        e0, e1 = dev.event(), dev.event()
        if tp_timer is not None:
            tp_timer("start")
        e0.record(stream)
        ttft = run_once()
        e1.record(stream)
        tp_ms = tp_timer("stop") if tp_timer is not None else None
        dev.sync()
        t = torch.tensor([e0.elapsed_ms(e1) if tp_ms is None else tp_ms], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
        n_gpus = world if tp_timer is None else int(os.environ.get("WORLD_SIZE", "1"))
        if rank == 0:
            tok = B * args.static_output * world
            line = {"metric": "output_tokens_per_s", "workload": args.workload, "batch": B,
                    "value": round(tok / (ms / 1000.0), 1), "unit": "tokens/s", "n_gpus": n_gpus,
                    "ms_total": round(ms, 2), "ttft_p50_s": round(statistics.median(ttft), 4) if ttft else None,
                    "dtype": args.dtype,
                    "config": {"model": args.model, "prompt": args.static_prompt, "output": args.static_output,
                               "parallelism": (f"tp{n_gpus} ({args.comm} collectives)" if tp_timer is not None
                                               else (f"dp{world}" if world > 1 else "tp1"))}}
            if args.workload == "shared-prefix":
                line["config"]["shared_prefix"] = args.shared_prefix
            if getattr(eng, "spec", None) is not None:
                st = eng.spec.stats
                line["speculative"] = {"draft": args.draft, "k": args.spec_k, "rounds": st["rounds"],
                                       "acceptance": round(eng.spec.acceptance_rate(), 4)}
            print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
