"""`rusteeze` command line: serve, generate, chat, benchmark, download, info,
validate, version.

Commands and flags follow crates/rusteeze-cli/src (lib.rs:26-70 global
`-c/--config` [RUSTEEZE_CONFIG], `-l/--log-level` [LOG_LEVEL], `--json`;
serve.rs:10-86, generate.rs:9-65, chat.rs:10-42, benchmark.rs:10-50,
download.rs:10-37, info.rs:11-15, validate.rs).  In the reference most of
these print canned data (serve never loads a model, serve.rs:139-170;
benchmark times sleep(10ms), benchmark.rs:97-138); here every command runs
the real engine.  `--model` takes a local HF-layout directory or a named
random-init preset (`llama-3-8b`, `mixtral-8x7b`, ...), since checkpoints
cannot be downloaded on an offline box.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from typing import List, Optional

from rusteeze_b200 import __version__

BANNER = f"rusteeze_b200 {__version__} -- Blackwell (sm_100a) LLM inference engine"


def _model_args(p: argparse.ArgumentParser, required: bool = True) -> None:
    # Every default is None: an option the user did not give leaves the config file's (or the
    # environment's) value in place, so precedence stays defaults < file < env < CLI.  The model
    # may come from -m, RUSTEEZE_MODEL or model.path / model.preset in the config file; commands
    # that need one check after the config is loaded.
    p.add_argument("-m", "--model", default=None,
                   help="HF-layout model directory or a random-init preset name")
    p.add_argument("--device", default=None)
    p.add_argument("--dtype", default=None)
    p.add_argument("--tensor-parallel-size", type=int, default=None)
    p.add_argument("--data-parallel-size", type=int, default=None,
                   help="serve: D engine replicas (one GPU each) behind a request router")
    p.add_argument("--router-policy", default=None,
                   choices=["least_loaded", "round_robin", "random", "prefix_affinity"])
    p.add_argument("--max-model-len", type=int, default=None)
    p.add_argument("--gpu-memory-utilization", type=float, default=None)
    p.add_argument("--quantization", default=None, choices=[None, "fp8_block", "fp8"])
    p.add_argument("--enforce-eager", action="store_true", default=None)
    p.add_argument("--kv-cache-dtype", default=None, choices=["auto", "fp8", "fp8_e4m3", "fp8_e5m2"],
                   help="paged KV cache element type (fp8: half the bytes per token)")
    p.add_argument("--seed", type=int, default=None)
    p.set_defaults(model_required=required)


def _overrides(a) -> dict:
    model = {"device": a.device, "dtype": a.dtype, "tensor_parallel_size": a.tensor_parallel_size,
             "data_parallel_size": a.data_parallel_size, "max_model_len": a.max_model_len, "seed": a.seed}
    if a.model is None and os.environ.get("RUSTEEZE_MODEL"):
        a.model = os.environ["RUSTEEZE_MODEL"]       # a directory or a preset name
    if a.model:
        if os.path.isdir(a.model):
            model["path"] = a.model
        else:
            model["preset"] = a.model
    if getattr(a, "quantization", None):
        model["quantization"] = {"method": "fp8_block"}
    eng = {"gpu_memory_utilization": a.gpu_memory_utilization, "enforce_eager": a.enforce_eager,
           "kv_cache_dtype": a.kv_cache_dtype}
    return {"model": model, "engine": eng, "server": {"router_policy": a.router_policy}}


def _load_config(a, extra: Optional[dict] = None):
    from rusteeze_b200.config.config import merge_dict
    from rusteeze_b200.config.loader import ConfigLoader
    ov = _overrides(a) if hasattr(a, "device") else {}
    if extra:
        ov = merge_dict(ov, extra)
    cfg = ConfigLoader(a.config).load(ov)
    if getattr(a, "model_required", False) and not (cfg.model.path or cfg.model.preset):
        raise SystemExit("rusteeze: a model is required: -m/--model, RUSTEEZE_MODEL, or model.path / "
                         "model.preset in the config file")
    return cfg


def _engine(cfg):
    if cfg.model.tensor_parallel_size > 1:
        from rusteeze_b200.parallel.launcher import TPEngineLauncher
        return TPEngineLauncher(cfg).engine()
    from rusteeze_b200.engine.llm_engine import LLMEngine
    return LLMEngine(cfg)


# ----------------------------------------------------------------------------- commands
def cmd_serve(a) -> int:
    from rusteeze_b200.api.server import serve
    extra = {"server": {"host": a.host, "port": a.port, "api_key": a.api_key, "metrics_port": a.metrics_port,
                        "cors": {"enabled": True} if a.cors else None,
                        "trust_request_chat_template": a.trust_request_chat_template or None},
             "engine": {"max_num_seqs": a.max_num_seqs, "block_size": a.block_size, "swap_space_gb": a.swap_space,
                        "enable_prefix_caching": a.enable_prefix_caching,
                        "enable_chunked_prefill": a.enable_chunked_prefill,
                        "max_num_batched_tokens": a.max_num_batched_tokens},
             "model": {"chat_template": a.chat_template, "trust_remote_code": a.trust_remote_code}}
    if a.speculative_method == "ngram":
        extra["engine"]["speculative"] = {"method": "ngram", "num_speculative_tokens": a.num_speculative_tokens,
                                          "ngram_max": a.ngram_max, "ngram_min": a.ngram_min}
    elif a.speculative_model:
        extra["engine"]["speculative"] = {"draft_preset" if not os.path.isdir(a.speculative_model) else "draft_model":
                                          a.speculative_model, "num_speculative_tokens": a.num_speculative_tokens}
    cfg = _load_config(a, extra)
    if not a.json:
        print(BANNER, file=sys.stderr)
        print(f"serving {cfg.model.served_name()} on {cfg.server.host}:{cfg.server.port} "
              f"(tp={cfg.model.tensor_parallel_size}, dp={cfg.model.data_parallel_size})", file=sys.stderr)
    serve(cfg, engine=None if cfg.model.data_parallel_size > 1 else _engine(cfg))
    return 0


def _sp_from(a, **kw):
    from rusteeze_b200.core.sampling_params import SamplingParams
    return SamplingParams(max_tokens=a.max_tokens, temperature=a.temperature, top_p=a.top_p,
                          top_k=a.top_k if getattr(a, "top_k", None) else -1,
                          repetition_penalty=getattr(a, "repetition_penalty", 1.0),
                          stop=getattr(a, "stop", None) or [], seed=getattr(a, "seed_sampling", None),
                          n=getattr(a, "n", 1), **kw)


def cmd_generate(a) -> int:
    cfg = _load_config(a)
    eng = _engine(cfg)
    prompts: List[str] = []
    if a.prompt:
        prompts.append(a.prompt)
    if a.file:
        with open(a.file) as f:
            prompts += [ln.rstrip("\n") for ln in f if ln.strip()]
    if not prompts:
        prompts = [sys.stdin.read()]
    kw = {}
    guided = {k: v for k, v in (("regex", a.regex), ("choice", a.choice or None)) if v}
    if a.json_schema:
        with open(a.json_schema) as f:
            guided["json_schema"] = json.load(f)
    if guided:
        from rusteeze_b200.core.sampling_params import GuidedDecodingParams
        kw["guided_decoding"] = GuidedDecodingParams(**guided)
    if a.beam_width:
        kw.update(use_beam_search=True, best_of=a.beam_width, length_penalty=a.length_penalty)
        a.temperature, a.top_p, a.top_k = 0.0, 1.0, None
    sp = _sp_from(a, **kw)
    results = []
    for i, p in enumerate(prompts):
        rid = f"gen-{i}"
        eng.add_request(rid, p, sp)
        text = ""
        while eng.has_unfinished_requests():
            for o in eng.step():
                if a.stream and not a.json:
                    sys.stdout.write(o.delta_text[0] if o.delta_text else "")
                    sys.stdout.flush()
                if o.finished:
                    results.append({"prompt": p, "outputs": [{"text": c.text, "token_ids": c.token_ids,
                                                              "finish_reason": c.finish_reason} for c in o.outputs],
                                    "ttft_s": o.metrics.ttft, "tpot_s": o.metrics.tpot})
        if a.stream and not a.json:
            print()
        elif not a.json:
            for c in results[-1]["outputs"]:
                print(c["text"])
    if a.json or a.output:
        s = json.dumps(results, indent=1)
        if a.output:
            with open(a.output, "w") as f:
                f.write(s)
        if a.json:
            print(s)
    return 0


def cmd_chat(a) -> int:
    from rusteeze_b200.tokenizer.chat_template import ChatTemplate
    cfg = _load_config(a, {"model": {"chat_template": a.chat_template}})
    eng = _engine(cfg)
    tmpl = ChatTemplate.for_model(cfg.model.served_name(), eng.tokenizer, a.chat_template)
    history = [{"role": "system", "content": a.system}] if a.system else []
    sp = _sp_from(a)
    print("chat with", cfg.model.served_name(), "-- /quit /clear /history /help", file=sys.stderr)
    turn = 0
    for line in sys.stdin:
        line = line.rstrip("\n")
        if not line:
            continue
        if line in ("/quit", "/exit"):
            break
        if line == "/clear":
            history = history[:1] if a.system else []
            continue
        if line == "/history":
            print(json.dumps(history, indent=1))
            continue
        if line == "/help":
            print("/quit /clear /history /help")
            continue
        history.append({"role": "user", "content": line})
        prompt = tmpl.apply(history)
        eng.add_request(f"chat-{turn}", None, sp, eng.tokenizer.encode(prompt, add_special_tokens=False)
                        or eng.tokenizer.encode(prompt))
        reply = ""
        while eng.has_unfinished_requests():
            for o in eng.step():
                d = o.delta_text[0] if o.delta_text else ""
                reply += d
                sys.stdout.write(d)
                sys.stdout.flush()
        print()
        history.append({"role": "assistant", "content": reply})
        turn += 1
    if a.save:
        with open(a.save, "w") as f:
            json.dump(history, f, indent=1)
    return 0


def cmd_benchmark(a) -> int:
    """Offline throughput/latency benchmark through the engine API: static
    batch of --num-prompts requests (--input-len random tokens, --output-len
    tokens with EOS ignored), at most --concurrency in flight; device-timed
    where the engine runs on CUDA.  Reports output tok/s, TTFT/TPOT p50/p99."""
    import numpy as np
    from rusteeze_b200.core.sampling_params import SamplingParams
    if a.url:
        # a running server over HTTP (streamed /v1/completions), no engine in this process
        import asyncio
        from rusteeze_b200.utils.http_bench import run_http_benchmark
        extra = {"temperature": a.url_temperature} if a.url_temperature is not None else {}
        if a.url_top_p is not None:
            extra["top_p"] = a.url_top_p
        res = asyncio.run(run_http_benchmark(a.url, a.served_model or a.model or "default", a.vocab_size,
                                             a.num_prompts, a.input_len, a.output_len, a.concurrency,
                                             a.request_rate, a.seed or 0, extra_body=extra or None))
        s = json.dumps(res, indent=None if a.json else 1)
        print(s)
        if a.output:
            with open(a.output, "w") as f:
                f.write(s)
        return 0 if res["failed"] == 0 else 1
    cfg = _load_config(a, {"engine": {"max_num_seqs": max(a.concurrency, 1),
                                      "max_num_batched_tokens": max(8192, a.concurrency)}})
    eng = _engine(cfg)
    V = eng.model_config.vocab_size
    rng = np.random.default_rng(a.seed)
    sp = SamplingParams(temperature=0.0, max_tokens=a.output_len, ignore_eos=True)

    def batch(n):
        return [rng.integers(0, V, a.input_len).tolist() for _ in range(n)]

    for p in batch(min(a.warmup, a.num_prompts)):
        eng.add_request(None, None, SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True), p)
    while eng.has_unfinished_requests():
        eng.step()
    prompts = batch(a.num_prompts)
    ttft, tpot, lat = [], [], []
    gen0 = eng.stats_counters["generation_tokens"]
    t0 = time.perf_counter()
    nxt = 0
    while nxt < len(prompts) or eng.has_unfinished_requests():
        while nxt < len(prompts) and len(eng.requests) < a.concurrency:
            eng.add_request(None, None, sp, prompts[nxt])
            nxt += 1
        for o in eng.step():
            if o.finished:
                ttft.append(o.metrics.ttft)
                if o.metrics.tpot is not None:
                    tpot.append(o.metrics.tpot)
                lat.append(o.metrics.e2e_latency)
    try:
        import torch
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    except Exception:  # noqa: BLE001
        pass
    dt = time.perf_counter() - t0
    gen = eng.stats_counters["generation_tokens"] - gen0

    def pct(x, q):
        return float(np.percentile(x, q)) if x else None

    res = {"model": cfg.model.served_name(), "num_prompts": a.num_prompts, "input_len": a.input_len,
           "output_len": a.output_len, "concurrency": a.concurrency, "duration_s": dt,
           "output_tokens_per_s": gen / dt, "requests_per_s": a.num_prompts / dt,
           "ttft_p50_ms": pct(ttft, 50) and pct(ttft, 50) * 1e3, "ttft_p99_ms": pct(ttft, 99) and pct(ttft, 99) * 1e3,
           "tpot_p50_ms": pct(tpot, 50) and pct(tpot, 50) * 1e3, "tpot_p99_ms": pct(tpot, 99) and pct(tpot, 99) * 1e3,
           "latency_p50_s": pct(lat, 50), "latency_p99_s": pct(lat, 99)}
    s = json.dumps(res, indent=None if a.json else 1)
    print(s)
    if a.output:
        with open(a.output, "w") as f:
            f.write(s)
    return 0


def cmd_download(a) -> int:
    try:
        from huggingface_hub import snapshot_download
    except ImportError:
        print("huggingface_hub is not installed; place an HF-layout directory (config.json + *.safetensors) "
              "locally and pass it with --model", file=sys.stderr)
        return 2
    patterns = None
    if a.weights_only:
        patterns = ["*.safetensors", "*.json"]
    if a.files:
        patterns = [x.strip() for x in a.files.split(",")]
    path = snapshot_download(a.model_id, revision=a.revision, local_dir=a.output, token=a.token,
                             allow_patterns=patterns)
    print(path)
    return 0


def cmd_info(a) -> int:
    from rusteeze_b200.models.config import ModelConfig, get_preset
    mc = ModelConfig.from_json_file(a.model) if os.path.isdir(a.model) else get_preset(a.model)
    n = mc.num_params()
    d = {"name": mc.name, "architecture": mc.architecture.value, "parameters": n,
         "parameters_billions": round(n / 1e9, 3), "layers": mc.num_hidden_layers, "hidden": mc.hidden_size,
         "heads": mc.num_attention_heads, "kv_heads": mc.num_key_value_heads, "head_dim": mc.head_dim,
         "intermediate": mc.intermediate_size, "vocab": mc.vocab_size, "context": mc.max_position_embeddings,
         "experts": mc.num_local_experts, "experts_per_token": mc.num_experts_per_tok,
         "bf16_weight_gib": round(n * 2 / 2 ** 30, 2), "kv_bytes_per_token_bf16": mc.kv_bytes_per_token(2)}
    if a.detailed:
        d["config"] = mc.to_hf_dict()
    print(json.dumps(d, indent=1))
    return 0


def cmd_validate(a) -> int:
    from rusteeze_b200.config.loader import ConfigLoader
    from rusteeze_b200.config.validation import collect_errors
    from rusteeze_b200.core.errors import ConfigError
    path = a.file or a.config
    try:
        cfg = ConfigLoader(path).load(validate=False)
    except ConfigError as e:
        print(json.dumps({"valid": False, "errors": [str(e)]}) if a.json else f"invalid: {e}")
        return 1
    errs = collect_errors(cfg)
    if a.json:
        print(json.dumps({"valid": not errs, "errors": errs}))
    else:
        print("configuration is valid" if not errs else "invalid:\n  - " + "\n  - ".join(errs))
    return 0 if not errs else 1


def cmd_quantize(a) -> int:
    """Writes an INT8 (per-channel), GPTQ or AWQ (grouped 4-bit) copy of a checkpoint or
    preset; GPTQ and AWQ calibrate on random token sequences unless a file of token-id
    lists (one JSON list per line) is given."""
    import numpy as np
    import torch
    from rusteeze_b200.models import int_quant as iq
    from rusteeze_b200.models.config import ModelConfig, get_preset
    from rusteeze_b200.models.loader import build_model
    is_dir = os.path.isdir(a.model)
    mc = ModelConfig.from_json_file(a.model) if is_dir else get_preset(a.model)
    if mc.is_moe:
        raise SystemExit("rusteeze quantize: MoE checkpoints are not quantized to integer formats")
    model = build_model(mc, dtype=torch.float32, model_dir=a.model if is_dir else None, seed=a.seed)
    if a.calibration:
        with open(a.calibration) as f:
            prompts = [json.loads(line) for line in f if line.strip()]
    else:
        rng = np.random.default_rng(a.seed)
        prompts = [rng.integers(0, mc.vocab_size, a.calibration_len).tolist() for _ in range(a.calibration_samples)]
    cfg = (iq.QuantConfig.int8() if a.method == "int8" else
           iq.QuantConfig(method=a.method, bits=4, group_size=a.group_size, act_order=a.act_order))
    cfg.exclude(a.exclude or [])
    stats = iq.QuantStats()
    iq.quantize_model_checkpoint(model, a.output, cfg, prompts, stats)
    if is_dir:                                    # keep the tokenizer with the weights
        import shutil
        for f in os.listdir(a.model):
            if f.startswith(("tokenizer", "special_tokens", "generation_config")):
                shutil.copy(os.path.join(a.model, f), os.path.join(a.output, f))
    d = {"output": a.output, "method": a.method, "layers": stats.layers_quantized,
         "compression": round(stats.compression_ratio(), 3), "mean_abs_error": stats.mean_error,
         "max_abs_error": stats.max_error}
    print(json.dumps(d) if a.json else "\n".join(f"{k}: {v}" for k, v in d.items()))
    return 0


def cmd_version(a) -> int:
    import platform
    d = {"version": __version__, "python": platform.python_version()}
    try:
        import torch
        d.update(torch=torch.__version__, cuda=torch.version.cuda)
    except Exception:  # noqa: BLE001
        pass
    print(json.dumps(d) if a.json else f"rusteeze_b200 {__version__}")
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="rusteeze", description=BANNER)
    ap.add_argument("-c", "--config", default=os.environ.get("RUSTEEZE_CONFIG"))
    ap.add_argument("-l", "--log-level", default=os.environ.get("LOG_LEVEL", "info"))
    ap.add_argument("--json", action="store_true", help="machine-readable output")
    sub = ap.add_subparsers(dest="cmd", required=True)

    s = sub.add_parser("serve", help="start the OpenAI-compatible server")
    _model_args(s)
    s.add_argument("--host", default=None)
    s.add_argument("-p", "--port", type=int, default=None)
    s.add_argument("--api-key", default=None)
    s.add_argument("--max-num-seqs", type=int, default=None)
    s.add_argument("--max-num-batched-tokens", type=int, default=None)
    s.add_argument("--enable-prefix-caching", action="store_true", default=None)
    s.add_argument("--enable-chunked-prefill", action="store_true", default=None)
    s.add_argument("--block-size", type=int, default=None)
    s.add_argument("--swap-space", type=float, default=None)
    s.add_argument("--cors", action="store_true", default=None)
    s.add_argument("--metrics-port", type=int, default=None)
    s.add_argument("--chat-template", default=None)
    s.add_argument("--trust-request-chat-template", action="store_true",
                   help="render a chat request's own Jinja chat_template (off: refused with 400)")
    s.add_argument("--trust-remote-code", action="store_true")
    s.add_argument("--pipeline-parallel-size", type=int, default=1)
    s.add_argument("--speculative-model", default=None)
    s.add_argument("--speculative-method", default="draft", choices=["draft", "ngram"],
                   help="ngram: prompt-lookup proposals, no draft model")
    s.add_argument("--num-speculative-tokens", type=int, default=4)
    s.add_argument("--ngram-max", type=int, default=4, help="longest suffix the ngram proposer looks up")
    s.add_argument("--ngram-min", type=int, default=1, help="shortest suffix the ngram proposer looks up")
    s.set_defaults(fn=cmd_serve)

    g = sub.add_parser("generate", help="offline generation")
    _model_args(g)
    g.add_argument("-p", "--prompt")
    g.add_argument("-f", "--file")
    g.add_argument("--max-tokens", type=int, default=256)
    g.add_argument("--temperature", type=float, default=1.0)
    g.add_argument("--top-p", type=float, default=1.0)
    g.add_argument("--top-k", type=int, default=None)
    g.add_argument("--repetition-penalty", type=float, default=1.0)
    g.add_argument("--stop", action="append", default=[])
    g.add_argument("--sampling-seed", dest="seed_sampling", type=int, default=None)
    g.add_argument("-n", type=int, default=1)
    g.add_argument("--beam-width", type=int, default=None, help="beam search with this many beams (n best returned)")
    g.add_argument("--length-penalty", type=float, default=1.0)
    g.add_argument("--regex", default=None, help="constrain the output to this regular expression")
    g.add_argument("--choice", action="append", default=[], help="constrain the output to one of these (repeatable)")
    g.add_argument("--json-schema", default=None, help="constrain the output to JSON valid for this schema file")
    g.add_argument("--stream", action="store_true")
    g.add_argument("-o", "--output")
    g.set_defaults(fn=cmd_generate)

    c = sub.add_parser("chat", help="interactive chat on stdin")
    _model_args(c)
    c.add_argument("--system")
    c.add_argument("--max-tokens", type=int, default=512)
    c.add_argument("--temperature", type=float, default=0.7)
    c.add_argument("--top-p", type=float, default=0.9)
    c.add_argument("--chat-template")
    c.add_argument("--save")
    c.set_defaults(fn=cmd_chat)

    b = sub.add_parser("benchmark", help="offline throughput / latency benchmark")
    _model_args(b)
    b.add_argument("-n", "--num-prompts", type=int, default=100)
    b.add_argument("--input-len", type=int, default=128)
    b.add_argument("--output-len", type=int, default=128)
    b.add_argument("--concurrency", type=int, default=1)
    b.add_argument("--warmup", type=int, default=3)
    b.add_argument("-o", "--output")
    b.add_argument("--url", default=None,
                   help="benchmark a running OpenAI-compatible server at this base URL over HTTP instead")
    b.add_argument("--request-rate", type=float, default=None, help="--url: Poisson arrivals per second")
    b.add_argument("--url-temperature", type=float, default=None, help="--url: sampling temperature (default greedy)")
    b.add_argument("--url-top-p", type=float, default=None, help="--url: top-p of the requests")
    b.add_argument("--served-model", default=None, help="--url: the model name sent in requests")
    b.add_argument("--vocab-size", type=int, default=32000, help="--url: range of the random prompt token ids")
    b.set_defaults(fn=cmd_benchmark)

    d = sub.add_parser("download", help="download an HF model snapshot (needs network)")
    d.add_argument("model_id")
    d.add_argument("--revision", default="main")
    d.add_argument("-o", "--output")
    d.add_argument("--token", default=os.environ.get("HF_TOKEN"))
    d.add_argument("--weights-only", action="store_true")
    d.add_argument("--files")
    d.add_argument("--resume", action="store_true")
    d.set_defaults(fn=cmd_download)

    i = sub.add_parser("info", help="model architecture summary")
    i.add_argument("model")
    i.add_argument("-d", "--detailed", action="store_true")
    i.set_defaults(fn=cmd_info)

    v = sub.add_parser("validate", help="validate a config file")
    v.add_argument("file", nargs="?")
    v.set_defaults(fn=cmd_validate)

    qz = sub.add_parser("quantize", help="write an INT8 / GPTQ / AWQ copy of a checkpoint")
    qz.add_argument("-m", "--model", required=True, help="HF-layout model directory or a preset name")
    qz.add_argument("-o", "--output", required=True)
    qz.add_argument("--method", default="gptq", choices=["int8", "gptq", "awq"])
    qz.add_argument("--group-size", type=int, default=128)
    qz.add_argument("--act-order", action="store_true", help="GPTQ: columns by decreasing Hessian diagonal")
    qz.add_argument("--calibration", default=None, help="file with one JSON list of token ids per line")
    qz.add_argument("--calibration-samples", type=int, default=32)
    qz.add_argument("--calibration-len", type=int, default=256)
    qz.add_argument("--exclude", nargs="*", help="layer names kept in full precision")
    qz.add_argument("--seed", type=int, default=0)
    qz.set_defaults(fn=cmd_quantize)

    ve = sub.add_parser("version")
    ve.set_defaults(fn=cmd_version)
    return ap


def main(argv: Optional[List[str]] = None) -> int:
    a = build_parser().parse_args(argv)
    from rusteeze_b200.metrics.logging_setup import init_logging
    init_logging(a.log_level)
    if getattr(a, "pipeline_parallel_size", 1) != 1:
        print("error: pipeline_parallel_size > 1 is not supported (use --tensor-parallel-size)", file=sys.stderr)
        return 2
    return a.fn(a)


if __name__ == "__main__":
    sys.exit(main())
