"""FP8 paged KV cache (e4m3 / e5m2): the codec, the oracle, the engine on CPU, and the
sm_100a kernels (RoPE + KV write, decode attention on fp8 pages, the bf16 scratch gather
that feeds prefill) against the fp32 oracle over the same cache bytes."""
import numpy as np
import pytest
import torch

from rusteeze_b200 import ops
from rusteeze_b200.config.config import Config
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.core.types import ModelArchitecture as A
from rusteeze_b200.engine.llm_engine import LLMEngine, kv_cache_dtype
from rusteeze_b200.models.config import tiny_variant
from rusteeze_b200.ops import reference as ref

FP8 = [torch.float8_e4m3fn, torch.float8_e5m2]
FP8_IDS = ["e4m3", "e5m2"]


def test_codec_saturates_rounds_and_scales():
    x = torch.tensor([1000.0, -1e6, 0.3, float("nan"), 3.0])
    e4 = ref.to_kv(x, torch.float8_e4m3fn).float()
    assert e4[0] == 448 and e4[1] == -448 and torch.isnan(e4[3])
    e5 = ref.to_kv(x, torch.float8_e5m2).float()
    assert e5[0] == 1024 and e5[1] == -57344
    # value / scale is stored: 3.0 / 0.5 = 6 (exact in both formats)
    assert float(ref.to_kv(x, torch.float8_e4m3fn, 0.5)[4].float()) == 6.0
    assert ref.to_kv(x, torch.bfloat16).dtype == torch.bfloat16


@pytest.mark.parametrize("dt", FP8, ids=FP8_IDS)
def test_oracle_reads_fp8_cache_with_scales(dt):
    """Attention over an fp8 cache with scales equals attention over a float cache holding
    the decoded values."""
    g = torch.Generator().manual_seed(0)
    nb, Hkv, D, Hq = 12, 2, 32, 4
    kf = torch.randn(nb, Hkv, 16, D, generator=g) * 3
    vf = torch.randn(nb, Hkv, 16, D, generator=g)
    ks, vs = 0.5, 2.0
    k8, v8 = ref.to_kv(kf, dt, ks), ref.to_kv(vf, dt, vs)
    kd, vd = k8.float() * ks, v8.float() * vs
    sl = torch.tensor([40, 70], dtype=torch.int32)
    bt = torch.tensor([[0, 1, 2, 0, 0], [3, 4, 5, 6, 7]], dtype=torch.int32)
    q = torch.randn(2 + 5, Hq, D, generator=g)
    qsl = torch.tensor([0, 2, 7], dtype=torch.int32)
    a = ref.paged_attention(q, k8, v8, qsl, sl, bt, D ** -0.5, k_scale=ks, v_scale=vs)
    b = ref.paged_attention(q, kd, vd, qsl, sl, bt, D ** -0.5)
    assert torch.allclose(a, b, atol=1e-5)


def _engine(kv: str, device="cpu", dtype="float32", mc=None, preemption_mode=None, **eng):
    cfg = Config()
    cfg.model.device = device
    cfg.model.dtype = dtype
    cfg.engine.kv_cache_dtype = kv
    if preemption_mode:
        cfg.engine.scheduling.preemption_mode = preemption_mode
    cfg.engine.num_gpu_blocks = eng.pop("num_gpu_blocks", 64)
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = eng.pop("max_num_batched_tokens", 96)
    cfg.engine.enable_chunked_prefill = True
    for k, v in eng.items():
        setattr(cfg.engine, k, v)
    return LLMEngine(cfg, model_config=mc or tiny_variant(A.LLAMA))


def _first_logprobs(eng, prompt, k=5):
    eng.add_request("probe", None, SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True, logprobs=k),
                    prompt)
    out = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            out = o
    return out.outputs[0].logprobs[0]


def test_kv_cache_dtype_names():
    assert kv_cache_dtype("auto", torch.bfloat16) is torch.bfloat16
    assert kv_cache_dtype("fp8", torch.bfloat16) is torch.float8_e4m3fn
    assert kv_cache_dtype("fp8_e4m3", torch.bfloat16) is torch.float8_e4m3fn
    assert kv_cache_dtype("fp8_e5m2", torch.float32) is torch.float8_e5m2


@pytest.mark.parametrize("kv", ["fp8_e4m3", "fp8_e5m2"])
def test_fp8_kv_engine_on_cpu_tracks_the_float_cache(kv):
    """The paged engine with an fp8 cache: first-step logprobs near the fp32-cache engine's,
    and a mixed workload with prefix caching and swap preemption (block copies and swaps
    of fp8 blocks) runs every request to the end."""
    mc = tiny_variant(A.LLAMA)
    p = np.random.default_rng(5).integers(0, mc.vocab_size, 60).tolist()
    base = _first_logprobs(_engine("auto", mc=mc), p)
    eng = _engine(kv, mc=mc)
    assert eng.runner.kv_cache.dtype == kv_cache_dtype(kv, torch.float32)
    got = _first_logprobs(eng, p)
    err = max(abs(got[t] - lp) for t, lp in base.items() if t in got)
    assert len(set(got) & set(base)) >= 4 and err < 0.1, err
    eng2 = _engine(kv, mc=mc, num_gpu_blocks=24, enable_prefix_caching=True, preemption_mode="swap")
    assert eng2.runner.cpu_cache is not None and eng2.runner.cpu_cache.dtype == eng2.runner.kv_cache.dtype
    rng = np.random.default_rng(9)
    shared = rng.integers(0, mc.vocab_size, 48).tolist()
    sp = SamplingParams(temperature=0.8, max_tokens=24, ignore_eos=True, seed=3)
    ids = [eng2.add_request(None, None, sp, shared + rng.integers(0, mc.vocab_size, int(n)).tolist()).request_id
           for n in (5, 30, 17, 60, 9, 44)]
    done = set()
    for _ in range(2000):
        if not eng2.has_unfinished_requests():
            break
        for o in eng2.step():
            if o.finished:
                done.add(o.request_id)
    assert done == set(ids)


def test_fp8_kv_cache_is_accepted_by_validation_and_cli():
    from rusteeze_b200.cli.main import build_parser
    from rusteeze_b200.config.validation import validate_config
    cfg = Config()
    for name in ("fp8", "fp8_e4m3", "fp8_e5m2"):
        cfg.engine.kv_cache_dtype = name
        validate_config(cfg)
    a = build_parser().parse_args(["generate", "-m", "tiny-llama", "--kv-cache-dtype", "fp8_e5m2", "-p", "x"])
    assert a.kv_cache_dtype == "fp8_e5m2"


# ----------------------------------------------------------------------------- GPU kernels
DEV = "cuda:0"


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.gpu
@pytest.mark.parametrize("dt", FP8, ids=FP8_IDS)
def test_rope_and_cache_writes_fp8(dt):
    T, Hq, Hkv, D = 37, 8, 2, 128
    g = torch.Generator().manual_seed(1)
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, generator=g) * 4).to(torch.bfloat16)
    pos = torch.randint(0, 500, (T,), generator=g)
    cs = ref.rope_cos_sin_cache(D, 512, 10000.0)
    slots = torch.randperm(20 * 16, generator=g)[:T]
    slots[3] = -1
    kc = torch.zeros(20, Hkv, 16, D, dtype=dt)
    vc = torch.zeros_like(kc)
    kd, vd = kc.view(torch.uint8).to(DEV).view(dt), vc.view(torch.uint8).to(DEV).view(dt)
    ops.rope_and_cache(qkv.clone().to(DEV), pos.to(DEV), cs.to(DEV), kd, vd, slots.to(DEV), Hq, Hkv, D, 0.5, 2.0)
    ops.rope_and_cache(qkv.clone(), pos, cs, kc, vc, slots, Hq, Hkv, D, 0.5, 2.0)
    # one rounding (fp32 -> fp8) in the kernel, two (fp32 -> bf16 -> fp8) in the oracle:
    # values agree within one fp8 step
    for got, want in ((kd, kc), (vd, vc)):
        g8, w8 = got.view(torch.uint8).cpu().view(dt).float(), want.float()
        step = w8.abs().clamp_min(2.0 ** -6) * (2.0 ** -3 if dt == torch.float8_e4m3fn else 2.0 ** -2)
        assert bool(((g8 - w8).abs() <= step + 1e-6).all())
        assert float((g8 == w8).float().mean()) > 0.97


def _fp8_cache(seq_lens, Hkv, D, dt, seed):
    g = torch.Generator().manual_seed(seed)
    nb = sum((l + 15) // 16 for l in seq_lens) + 4
    kf = torch.randn(nb, Hkv, 16, D, generator=g) * 2
    vf = torch.randn(nb, Hkv, 16, D, generator=g)
    perm = torch.randperm(nb, generator=g)
    mb = max((l + 15) // 16 for l in seq_lens) + 1
    bt = torch.zeros(len(seq_lens), mb, dtype=torch.int32)
    c = 0
    for i, l in enumerate(seq_lens):
        n = (l + 15) // 16
        bt[i, :n] = perm[c:c + n].int()
        c += n
    return ref.to_kv(kf, dt, 0.5), ref.to_kv(vf, dt, 2.0), bt


def _dev8(t):
    return t.view(torch.uint8).to(DEV).view(t.dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("dt", FP8, ids=FP8_IDS)
@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (8, 8, 128), (16, 2, 64), (8, 2, 256)])
@pytest.mark.parametrize("splits", [1, 4])
def test_decode_attention_on_fp8_pages(dt, Hq, Hkv, D, splits):
    seq_lens = [1, 17, 100, 511, 1030, 64]
    k8, v8, bt = _fp8_cache(seq_lens, Hkv, D, dt, seed=3)
    S = len(seq_lens)
    q = torch.randn(S, Hq, D, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    qsl = torch.arange(S + 1, dtype=torch.int32)
    want = ref.paged_attention(q, k8, v8, qsl, sl, bt, D ** -0.5, k_scale=0.5, v_scale=2.0)
    ws = torch.empty(S * Hq * splits * (D + 2), device=DEV)
    out = torch.zeros(q.shape, device=DEV, dtype=torch.bfloat16)
    ops.cuda_ext().decode_attention(out, q.to(DEV), _dev8(k8), _dev8(v8), sl.to(DEV), bt.to(DEV), ws, S,
                                    D ** -0.5, 0, 0.0, splits, None, 0.5, 2.0)
    assert _rel(out, want) < 1e-2
    assert int(ops.cuda_ext().status()[0]) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dt", FP8, ids=FP8_IDS)
def test_paged_attention_mixed_batch_on_fp8_cache(dt):
    """Decode rows read the fp8 pages; prefill and chunked rows read the bf16 scratch gather;
    with ALiBi and a window to cover the variants."""
    from rusteeze_b200.models.decoder import AttentionMetadata
    Hq, Hkv, D = 32, 8, 128
    specs = [(90, 1), (300, 1), (130, 1), (77, 77), (700, 200)]      # 3 decodes, then prefills
    seq_lens = [s for s, _ in specs]
    q_lens = [x for _, x in specs]
    k8, v8, bt = _fp8_cache(seq_lens, Hkv, D, dt, seed=8)
    T = sum(q_lens)
    q = torch.randn(T, Hq, D, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    qsl = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    slopes = ref.alibi_slopes(Hq)
    for window, alibi in ((0, None), (60, slopes)):
        want = ref.paged_attention(q, k8, v8, qsl, sl, bt, D ** -0.5, window or None, None, alibi, 0.5, 2.0)
        nd = 3
        meta = AttentionMetadata(num_seqs=5, num_tokens=T, num_decode_seqs=nd, query_start_loc=qsl.to(DEV),
                                 seq_lens=sl.to(DEV), block_tables=bt.to(DEV),
                                 slot_mapping=torch.full((T,), -1, dtype=torch.int64, device=DEV),
                                 max_query_len=max(q_lens), max_seq_len=max(seq_lens), decode_num_splits=2,
                                 decode_workspace=torch.empty(nd * Hq * 2 * (D + 2), device=DEV),
                                 prefill_kv_blocks=sum((l + 15) // 16 for l in seq_lens[nd:]))
        out = ops.paged_attention(q.to(DEV), _dev8(k8), _dev8(v8), meta, D ** -0.5, window or None, None,
                                  None if alibi is None else alibi.to(DEV), 0.5, 2.0)
        assert _rel(out, want) < 1.5e-2, window
    assert int(ops.cuda_ext().status()[0]) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("kv,fmt,tol", [("fp8_e4m3", None, 0.15), ("fp8_e5m2", None, 0.25),
                                        ("fp8_e4m3", "ue8m0", 0.8)])
def test_fp8_kv_engine_on_gpu_tracks_the_fp32_oracle(kv, fmt, tol):
    """Engine on the GPU with an fp8 cache (bf16 weights, or MXFP8 weights): the first step's
    top-5 logprobs against the dense fp32 oracle on the unquantised weights, then greedy
    decoding through the CUDA graphs."""
    from rusteeze_b200.config.config import QuantizationConfig
    from rusteeze_b200.models.loader import build_model, to_cpu_fp32
    from rusteeze_b200.models.naive import naive_logits
    mc = tiny_variant(A.LLAMA, hidden_size=512, intermediate_size=1024, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, vocab_size=32000)
    p = np.random.default_rng(3).integers(0, mc.vocab_size, 50).tolist()
    # the engine's own random init (bf16 on the device, seed 0), run in fp32 on the CPU
    m = build_model(mc, dtype=torch.bfloat16, device=DEV, seed=0)
    want = torch.log_softmax(naive_logits(to_cpu_fp32(m), p)[-1].double(), -1)
    del m
    cfg = Config()
    cfg.model.device = DEV
    cfg.model.seed = 0
    cfg.engine.kv_cache_dtype = kv
    cfg.engine.num_gpu_blocks = 64
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 256
    if fmt:
        cfg.model.quantization = QuantizationConfig(method="fp8_block", scale_format=fmt)
    eng = LLMEngine(cfg, model_config=mc)
    top = _first_logprobs(eng, p)
    err = max(abs(lp - float(want[t])) for t, lp in top.items())
    assert err < tol, err
    sp = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True)
    for n in (7, 40, 90):
        eng.add_request(None, None, sp, (p * 2)[:n])
    outs = []
    while eng.has_unfinished_requests():
        outs += [o for o in eng.step() if o.finished]
    assert len(outs) == 3 and all(len(o.outputs[0].token_ids) == 24 for o in outs)
    assert int(ops.cuda_ext().status()[0]) == 0


def test_fp8_kv_with_speculative_decoding_matches_the_plain_fp8_engine():
    """Speculative verify reads the fp8 cache through the multi-token (prefill) path; greedy
    output equals the non-speculative engine on the same fp8 cache, and a self-draft
    accepts every proposal."""
    from rusteeze_b200.config.config import SpeculativeSection
    mc = tiny_variant(A.LLAMA)
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, mc.vocab_size, int(n)).tolist() for n in (20, 45)]

    def run(eng):
        sp = SamplingParams(temperature=0.0, max_tokens=9, ignore_eos=True)
        ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
        done = {}
        while eng.has_unfinished_requests():
            for o in eng.step():
                if o.finished:
                    done[o.request_id] = o.outputs[0].token_ids
        return [done[i] for i in ids]

    plain = run(_engine("fp8_e4m3", mc=mc))
    eng = _engine("fp8_e4m3", mc=mc, speculative=SpeculativeSection(num_speculative_tokens=3))
    assert run(eng) == plain
    assert eng.spec.stats["accepted"] == eng.spec.stats["proposed"] > 0


@pytest.mark.timeout(300)
def test_fp8_kv_tp2_gloo_matches_single_process():
    """fp8 caches in every rank's runner (the worker's included): a TP2 engine's greedy
    tokens equal the single-process engine's on the same fp8 cache format."""
    from rusteeze_b200.models.config import ModelConfig
    from rusteeze_b200.parallel.launcher import TPEngineLauncher
    mc = ModelConfig(name="tp-tiny", hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, vocab_size=1000, rms_norm_eps=1e-5,
                     max_position_embeddings=512)

    def cfg(tp):
        c = Config()
        c.model.device, c.model.dtype, c.model.tensor_parallel_size = "cpu", "float32", tp
        c.engine.num_gpu_blocks, c.engine.max_num_seqs, c.engine.max_num_batched_tokens = 96, 4, 128
        c.engine.enable_chunked_prefill, c.engine.comm_backend = True, "nccl"
        c.engine.kv_cache_dtype = "fp8_e5m2"
        return c

    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, 1000, int(n)).tolist() for n in (30, 70)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)

    def run(eng):
        ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
        done = {}
        while eng.has_unfinished_requests():
            for o in eng.step():
                if o.finished:
                    done[o.request_id] = o.outputs[0].token_ids
        return [done[i] for i in ids]

    ref = run(LLMEngine(cfg(1), model_config=mc))
    launcher = TPEngineLauncher(cfg(2), model_config=mc, device_type="cpu")
    try:
        eng = launcher.engine()
        assert eng.runner.runner.kv_cache.dtype == torch.float8_e5m2     # rank 0's runner under the executor
        got = run(eng)
    finally:
        launcher.shutdown()
    assert got == ref
