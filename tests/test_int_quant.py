"""Integer weight quantization: codecs, GPTQ / AWQ / SmoothQuant against their defining
properties, the GPTQ / AWQ / INT8 checkpoint layouts, and quantized checkpoints loaded by
the engine (dequantized at load)."""
import json
import os

import numpy as np
import pytest
import torch

from rusteeze_b200.models import int_quant as iq
from rusteeze_b200.models.config import tiny_variant
from rusteeze_b200.core.types import ModelArchitecture as A


def _g(seed):
    return torch.Generator().manual_seed(seed)


def test_int8_per_channel_and_per_tensor_round_trip():
    w = torch.randn(64, 256, generator=_g(0)) * torch.linspace(0.01, 3, 64).unsqueeze(1)
    for per_channel in (True, False):
        for sym in (True, False):
            q, st = iq.quantize_int8(w, per_channel, sym)
            assert q.dtype == (torch.int8 if sym else torch.uint8)
            err = (iq.dequantize_int8(q, st) - w).abs()
            assert bool((err <= st.scales * 0.5 + 1e-6).all()), (per_channel, sym)


@pytest.mark.parametrize("bits,sym", [(4, False), (4, True), (8, False)])
def test_grouped_round_trip_error_is_half_a_step(bits, sym):
    w = torch.randn(32, 512, generator=_g(1))
    q, st = iq.quantize_grouped(w, bits, 128, sym)
    lo, hi = iq._qrange(bits, sym)
    assert int(q.min()) >= lo and int(q.max()) <= hi
    err = (iq.dequantize_grouped(q, st) - w).abs().view(32, 4, 128)
    assert bool((err <= st.scales.view(32, 4, 1) * 0.5 + 1e-6).all())
    with pytest.raises(ValueError):
        iq.quantize_grouped(torch.zeros(4, 100), 4, 128)


def test_int4_pack_unpack_is_identity():
    c = torch.randint(0, 16, (7, 64), generator=_g(2), dtype=torch.uint8)
    p = iq.pack_int4(c)
    assert p.shape == (7, 32) and torch.equal(iq.unpack_int4(p), c)


@pytest.mark.parametrize("cfg,tol", [(iq.QuantConfig.int8(), 0.01), (iq.QuantConfig.int4(64), 0.12),
                                     (iq.QuantConfig(method="int4", bits=4, group_size=64, symmetric=True), 0.15)])
def test_quantized_linear_tracks_the_float_layer(cfg, tol):
    w = torch.randn(96, 256, generator=_g(3)) * 0.05
    b = torch.randn(96, generator=_g(4))
    x = torch.randn(10, 256, generator=_g(5))
    ql = iq.QuantizedLinear.from_float(w, b, cfg)
    ref = x @ w.t() + b
    rel = float((ql(x) - ref).norm() / ref.norm())
    assert rel < tol, rel
    assert ql.memory_savings() > (0.4 if cfg.bits == 8 else 0.65)


def test_quant_config_presets_and_exclusions():
    c = iq.QuantConfig.gptq(4, 64).exclude(["lm_head"])
    assert c.method == "gptq" and c.bits == 4 and c.group_size == 64 and c.skips("model.lm_head")
    assert not c.skips("model.layers.0.mlp.down_proj")
    assert iq.QuantConfig.awq().with_group_size(32).group_size == 32
    with pytest.raises(ValueError):
        iq.QuantConfig(method="int3")


def _correlated_inputs(T, K, seed):
    g = _g(seed)
    z = torch.randn(T, K // 4, generator=g)
    mix = torch.randn(K // 4, K, generator=g)
    return z @ mix + 0.05 * torch.randn(T, K, generator=g)


def test_gptq_with_an_identity_hessian_is_round_to_nearest():
    w = torch.randn(16, 256, generator=_g(6))
    codes, scales, zeros, g_idx = iq.gptq_quantize(w, torch.eye(256), bits=4, group_size=64, damp_percent=0.0)
    q, st = iq.quantize_grouped(w, 4, 64, symmetric=False)
    assert torch.equal(codes, q)
    assert torch.allclose(scales, st.scales) and torch.allclose(zeros, st.zero_points)
    assert torch.equal(g_idx, (torch.arange(256) // 64).int())


@pytest.mark.parametrize("act_order", [False, True])
def test_gptq_beats_round_to_nearest_on_correlated_inputs(act_order):
    K = 256
    w = torch.randn(64, K, generator=_g(7)) * 0.1
    x = _correlated_inputs(2048, K, 8)
    codes, scales, zeros, g_idx = iq.gptq_quantize(w, iq.hessian(x), 4, 64, act_order=act_order)
    w_gptq = iq.dequantize_gptq(codes, scales, zeros, g_idx)
    q, st = iq.quantize_grouped(w, 4, 64)
    w_rtn = iq.dequantize_grouped(q, st)
    ref = x @ w.t()
    e_gptq = float((x @ w_gptq.t() - ref).pow(2).mean())
    e_rtn = float((x @ w_rtn.t() - ref).pow(2).mean())
    assert e_gptq < 0.7 * e_rtn, (e_gptq, e_rtn)


def test_awq_scales_never_lose_to_plain_grouped_quantization():
    K = 256
    w = torch.randn(64, K, generator=_g(9)) * 0.1
    x = torch.randn(512, K, generator=_g(10))
    x[:, :8] *= 30.0                       # salient input channels
    s, a = iq.awq_search_scales(w, x, 4, 64)
    q, st = iq.quantize_grouped(w * s, 4, 64)
    w_awq = iq.dequantize_grouped(q, st) / s
    q0, st0 = iq.quantize_grouped(w, 4, 64)
    w_rtn = iq.dequantize_grouped(q0, st0)
    ref = x @ w.t()
    e_awq = float((x @ w_awq.t() - ref).pow(2).mean())
    e_rtn = float((x @ w_rtn.t() - ref).pow(2).mean())
    assert a > 0 and e_awq < e_rtn
    norm = torch.rand(K, generator=_g(11)) + 0.5
    assert torch.allclose(iq.fold_input_scale(norm, s), norm / s)


def test_smoothquant_keeps_the_product():
    K = 128
    x = torch.randn(32, K, generator=_g(12))
    x[:, 3] *= 50
    ws = [torch.randn(40, K, generator=_g(13)), torch.randn(24, K, generator=_g(14))]
    s = iq.smoothquant_scales(x.abs().amax(0), ws, alpha=0.5)
    norm = torch.ones(K)
    n2, ws2 = iq.apply_smoothing(norm, ws, s)
    for w, w2 in zip(ws, ws2):
        assert torch.allclose((x * n2) @ w2.t(), x @ w.t(), rtol=1e-4, atol=1e-3)
    assert float((x * n2).abs().amax(0).max()) < float(x.abs().amax(0).max())


def test_gptq_and_awq_layouts_round_trip():
    N, K, g = 64, 256, 64
    codes = torch.randint(0, 16, (N, K), generator=_g(15), dtype=torch.uint8)
    scales = torch.rand(N, K // g, generator=_g(16)) * 0.1 + 0.01
    zeros = torch.randint(0, 16, (N, K // g), generator=_g(17)).float()
    g_idx = (torch.arange(K) // g).int()
    want = iq.dequantize_gptq(codes, scales.half().float(), zeros, g_idx)
    for v2 in (False, True):
        # the v1 layout stores zero - 1 in 4 bits: a zero point of 0 cannot be written (it
        # reads back as 16), which is why gptq_v2 exists; v1 is checked on zeros 1..15
        z = zeros if v2 else zeros.clamp_min(1)
        want = iq.dequantize_gptq(codes, scales.half().float(), z, g_idx)
        t = iq.pack_gptq(codes, scales, z, g_idx, 4, v2=v2)
        assert t["qweight"].shape == (K // 8, N) and t["qweight"].dtype == torch.int32
        assert t["qzeros"].shape == (K // g, N // 8)
        assert torch.allclose(iq.unpack_gptq(t, 4, v2=v2), want)
    want = iq.dequantize_gptq(codes, scales.half().float(), zeros, g_idx)
    t = iq.pack_awq(codes, scales, zeros, 4)
    assert t["qweight"].shape == (K, N // 8)
    assert torch.allclose(iq.unpack_awq(t, 4), want)
    # the interleaved AWQ order: output 1 sits in slot 4 (bits 16..19) of the first word
    one = torch.zeros(N, K, dtype=torch.uint8)
    one[1, 0] = 9
    w0 = int(iq.pack_awq(one, scales, torch.zeros_like(zeros), 4)["qweight"][0, 0])
    assert (w0 >> 16) & 0xF == 9


def test_calibration_collector_statistics():
    col = iq.CalibrationCollector(keep_inputs=True, max_rows=5)
    col.record("a", torch.tensor([[1.0, -4.0], [2.0, 0.0]]))
    col.record("a", torch.tensor([[-3.0, 1.0], [0.0, 0.0], [1.0, 1.0], [9.0, 9.0]]))
    st = col.get_stats("a")
    assert st["absmax"].tolist() == [9.0, 9.0] and int(st["count"]) == 6
    assert col.layer_inputs("a").shape == (5, 2) and col.get_stats("b") is None


@pytest.mark.parametrize("method,tol", [("int8", 0.02), ("gptq", 0.2), ("awq", 0.2)])
def test_quantized_checkpoint_loads_through_the_engine(tmp_path, method, tol):
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.core.sampling_params import SamplingParams
    from rusteeze_b200.engine.llm_engine import LLMEngine
    from rusteeze_b200.models.loader import build_model, checkpoint_quantization
    from rusteeze_b200.models.naive import naive_logits
    mc = tiny_variant(A.LLAMA, hidden_size=128, intermediate_size=256)
    model = build_model(mc, dtype=torch.float32, seed=5)
    rng = np.random.default_rng(0)
    calib = [rng.integers(0, mc.vocab_size, 48).tolist() for _ in range(4)]
    cfg = iq.QuantConfig.int8() if method == "int8" else iq.QuantConfig(method=method, bits=4, group_size=64)
    stats = iq.QuantStats()
    out = iq.quantize_model_checkpoint(model, str(tmp_path), cfg, calib, stats)
    assert stats.layers_quantized == 7 * mc.num_hidden_layers and stats.compression_ratio() > 1.5
    assert any(k.endswith(".qweight") for k in out) == (method != "int8")
    hf = json.load(open(os.path.join(tmp_path, "config.json")))
    assert hf["quantization_config"]["quant_method"] == method
    assert checkpoint_quantization(str(tmp_path))["quant_method"] == method
    # the dequantized model stays close to the float one
    loaded = build_model(mc, dtype=torch.float32, model_dir=str(tmp_path))
    p = calib[0]
    a, b = naive_logits(model, p), naive_logits(loaded, p)
    rel = float((a - b).norm() / a.norm())
    assert rel < tol, rel
    # and the engine serves it
    c = Config()
    c.model.device, c.model.dtype, c.model.path = "cpu", "float32", str(tmp_path)
    c.engine.num_gpu_blocks, c.engine.max_num_seqs = 64, 4
    eng = LLMEngine(c)
    eng.add_request("r", None, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True), p)
    toks = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                toks = o.outputs[0].token_ids
    assert toks is not None and len(toks) == 6


def test_cli_quantize_writes_a_servable_checkpoint(tmp_path):
    """`rusteeze quantize` on a preset: a GPTQ checkpoint that `rusteeze info` reads and the
    engine generates from."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=root)
    out = tmp_path / "q"
    r = subprocess.run([sys.executable, "-m", "rusteeze_b200", "--json", "quantize", "-m", "tiny-llama", "-o",
                        str(out), "--method", "gptq", "--group-size", "64", "--calibration-samples", "2",
                        "--calibration-len", "32"], capture_output=True, text=True, timeout=600, cwd=root, env=env)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["method"] == "gptq" and d["layers"] == 14 and d["compression"] > 2
    r = subprocess.run([sys.executable, "-m", "rusteeze_b200", "generate", "-m", str(out), "--device", "cpu",
                        "--dtype", "float32", "-p", "hello", "--max-tokens", "4"], capture_output=True, text=True,
                       timeout=600, cwd=root, env=env)
    assert r.returncode == 0, r.stderr
