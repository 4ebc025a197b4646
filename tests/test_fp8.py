"""FP8 block-scaled path: codec vs torch float8, quantised model on CPU
(oracle math), and the sm_100a kernels (GPU) vs the dequantise-then-matmul
fp32 oracle."""
import dataclasses

import pytest
import torch

from rusteeze_b200 import ops
from rusteeze_b200.models.config import ModelConfig
from rusteeze_b200.ops import reference as ref


def test_weight_and_activation_codec_roundtrip():
    torch.manual_seed(0)
    w = torch.randn(300, 512) * 0.05
    q, s = ref.quant_fp8_weight(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (3, 4)
    deq = (torch.zeros(384, 512).index_copy_(0, torch.arange(300), q.float())
           .view(3, 128, 4, 128) * s[:, None, :, None]).view(384, 512)[:300]
    assert ((deq - w).abs().max() / w.abs().max()) < 0.07          # e4m3: 3 mantissa bits
    x = torch.randn(7, 256)
    xq, xs = ref.quant_fp8_act(x)
    assert xs.shape == (7, 2)
    back = xq.float().view(7, 2, 128) * xs.unsqueeze(-1)
    assert torch.allclose(back.view(7, 256), x, rtol=0.07, atol=1e-3)


def test_fp8_model_cpu_tracks_bf16_model():
    from rusteeze_b200.models.loader import build_model
    from rusteeze_b200.models.naive import naive_logits
    from rusteeze_b200.models.quant import quantize_model_fp8
    from rusteeze_b200.models.decoder import AttentionMetadata
    mc = ModelConfig(name="fp8-tiny", hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, vocab_size=1024, max_position_embeddings=512)
    m = build_model(mc, dtype=torch.float32, seed=1)
    p = list(range(3, 40))
    ref_logits = naive_logits(m, p)[-1]
    quantize_model_fp8(m)
    # paged forward of the quantised model (1 sequence, 1 block table)
    T = len(p)
    nb = (T + 15) // 16
    kv = [(torch.zeros(8, m.hkv, 16, mc.head_dim), torch.zeros(8, m.hkv, 16, mc.head_dim))
          for _ in range(mc.num_hidden_layers)]
    meta = AttentionMetadata(num_seqs=1, num_tokens=T, num_decode_seqs=0,
                             query_start_loc=torch.tensor([0, T], dtype=torch.int32),
                             seq_lens=torch.tensor([T], dtype=torch.int32),
                             block_tables=torch.arange(nb, dtype=torch.int32).view(1, nb),
                             slot_mapping=torch.arange(T), max_query_len=T)
    h = m(torch.tensor(p), torch.arange(T), meta, kv)
    logits = m.compute_logits(h[-1:])[0]
    cos = torch.nn.functional.cosine_similarity(logits, ref_logits, dim=0)
    assert cos > 0.99, float(cos)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 256, 256), (7, 4096, 4096), (256, 6144, 4096), (1300, 4096, 14336),
                                   (64, 1024, 512), (129, 128256 // 8 - 32, 1024)])
def test_gemm_fp8_vs_oracle(M, N, K):
    torch.manual_seed(M + N)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda") * 0.02
    wq, ws = ref.quant_fp8_weight(w)
    y = ops.linear_fp8(x, wq, ws)
    xq, xs = ops.quant_fp8_act(x)
    r = ref.fp8_block_gemm(xq.cpu(), xs.t().cpu(), wq.cpu(), ws.cpu())
    err = ((y.float().cpu() - r).norm() / r.norm()).item()
    assert err < 1e-2, err
    torch.cuda.synchronize()
    assert int(ops.cuda_ext().status()[0]) == 0


@pytest.mark.gpu
def test_quant_act_kernel_matches_reference():
    x = torch.randn(33, 1024, device="cuda", dtype=torch.bfloat16) * 3
    q, s = ops.quant_fp8_act(x)
    qr, sr = ref.quant_fp8_act(x.cpu())
    assert torch.allclose(s.t().cpu(), sr, rtol=1e-6)
    assert (q.float().cpu() - qr.float()).abs().max() <= 1.0 * qr.float().abs().max() * 0.07


@pytest.mark.gpu
@pytest.mark.parametrize("ks", [1, 4])
def test_gemm_fp8_silu_and_splitk(ks):
    torch.manual_seed(7)
    M, I, K = 200, 512, 2048
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wg = torch.randn(I, K, device="cuda") * 0.03
    wu = torch.randn(I, K, device="cuda") * 0.03
    wi = ops.interleave_gate_up(torch.cat([wg, wu]).to(torch.bfloat16)).float()
    wq, ws = ref.quant_fp8_weight(wi)
    xq, xs = ops.quant_fp8_act(x)
    out = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    ops.cuda_ext().gemm_fp8_block(out, xq, xs, wq, ws, None, None, 1, ks)
    full = ref.fp8_block_gemm(xq.cpu(), xs.t().cpu(), wq.cpu(), ws.cpu()).view(M, I // 64, 2, 64)
    r = (torch.nn.functional.silu(full[:, :, 0]) * full[:, :, 1]).reshape(M, I)
    err = ((out.float().cpu() - r).norm() / r.norm()).item()
    assert err < 1.5e-2, err
    y = torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    res = torch.randn(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    ops.cuda_ext().gemm_fp8_block(y, xq, xs, wq, ws, None, res, 0, ks)
    r2 = ref.fp8_block_gemm(xq.cpu(), xs.t().cpu(), wq.cpu(), ws.cpu()) + res.float().cpu()
    assert ((y.float().cpu() - r2).norm() / r2.norm()).item() < 1e-2


@pytest.mark.gpu
def test_fp8_engine_llama3_shapes_runs():
    from rusteeze_b200.config.config import Config, QuantizationConfig
    from rusteeze_b200.core.sampling_params import SamplingParams
    from rusteeze_b200.engine.llm_engine import LLMEngine
    from rusteeze_b200.models.config import get_preset
    mc = dataclasses.replace(get_preset("llama-3-8b"), num_hidden_layers=2)
    cfg = Config()
    cfg.model.device = "cuda:0"
    cfg.model.quantization = QuantizationConfig(method="fp8_block")
    cfg.engine.num_gpu_blocks = 256
    cfg.engine.max_num_seqs = 8
    cfg.engine.max_num_batched_tokens = 512
    eng = LLMEngine(cfg, model_config=mc)
    eng.add_request("a", None, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True), list(range(5, 90)))
    out = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            out = o
    assert len(out.outputs[0].token_ids) == 6


# ----------------------------------------------------------------------------- MXFP8 (UE8M0 scales)
def test_ue8m0_codec_and_scale_chunks():
    torch.manual_seed(3)
    w = torch.randn(256, 384) * 0.03
    q, s = ref.quant_mxf8_weight(w)
    assert torch.equal(s, ref.pow2_ceil(s))                      # powers of two
    assert (q.float().abs().amax() <= 448).item()
    deq = (q.float().view(2, 128, 3, 128) * s[:, None, :, None]).view(256, 384)
    assert ((deq - w).abs().max() / w.abs().max()) < 0.13          # up to one extra bit lost to the pow2 scale
    ch = ref.pack_block_scales_ue8m0(s)
    assert ch.shape == (2, 3, 512) and (ch[0, 1] == ch[0, 1, 0]).all()
    assert torch.equal(torch.ldexp(torch.ones(()), ch[1, 2, 0].long() - 127), s[1, 2])
    x = torch.randn(200, 256) * 3
    xq, xs = ref.quant_mxf8_act(x)
    sfa = ref.pack_act_scales_ue8m0(xs)
    assert sfa.shape == (2, 2, 512)
    off = (71 % 32) * 16 + (71 // 32) * 4                            # x row 199 = block 1, in-block row 71
    want = (torch.log2(xs[199]).round().long() + 127).to(torch.uint8)
    assert torch.equal(sfa[1, :, off], want) and torch.equal(sfa[1, :, off + 3], want)
    assert torch.equal(ref.unpack_act_scales_ue8m0(sfa, 200, 256), xs)
    assert int(sfa[1, 0, (127 % 32) * 16 + (127 // 32) * 4]) == 127   # padded row: neutral scale


def test_fp32_scale_format_model_cpu():
    from rusteeze_b200.models.loader import build_model
    from rusteeze_b200.models.quant import quantize_model_fp8
    mc = ModelConfig(name="fp8-tiny", hidden_size=256, intermediate_size=512, num_hidden_layers=1,
                     num_attention_heads=4, num_key_value_heads=2, vocab_size=1024, max_position_embeddings=512)
    m = build_model(mc, dtype=torch.float32, seed=1)
    quantize_model_fp8(m, "fp32")
    assert getattr(m.layers[0], "qkv_sf", None) is None and m.fp8_format == "fp32"
    m2 = build_model(mc, dtype=torch.float32, seed=1)
    quantize_model_fp8(m2)
    assert m2.layers[0].qkv_sf.dtype == torch.uint8 and m2.fp8_format == "ue8m0"


@pytest.mark.gpu
def test_quant_mxf8_act_kernel_matches_reference():
    torch.manual_seed(5)
    x = (torch.randn(300, 1024, device="cuda") * 2).to(torch.bfloat16)
    x[7, :128] = 0                                                   # all-zero block
    q, sfa = ops.quant_mxf8_act(x)
    qr, sr = ref.quant_mxf8_act(x.cpu())
    assert torch.equal(ref.unpack_act_scales_ue8m0(sfa.cpu(), 300, 1024)[torch.arange(300) != 7],
                       sr[torch.arange(300) != 7])
    assert torch.equal(q.cpu().view(torch.uint8)[torch.arange(300) != 7], qr.view(torch.uint8)[torch.arange(300) != 7])
    assert torch.equal(sfa.cpu()[2, :, (300 % 128 + 1) % 32 * 16 + (300 % 128 + 1) // 32 * 4],
                       torch.full((8,), 127, dtype=torch.uint8))     # padded row 301 -> neutral


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,bn,ks", [(1, 256, 256, 128, 1), (7, 4096, 4096, 256, 1), (200, 6144, 4096, 128, 1),
                                         (200, 6144, 4096, 256, 1), (1300, 4096, 14336, 256, 1),
                                         (64, 1024, 512, 128, 2), (129, 16000, 1024, 128, 1),
                                         (300, 2048, 4096, 256, 4), (1256, 28672, 4096, 0, 0)])
def test_gemm_mxf8_vs_oracle(M, N, K, bn, ks):
    torch.manual_seed(M + N + bn)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda") * 0.02
    wq, ws = ref.quant_mxf8_weight(w)
    wsf = ref.pack_block_scales_ue8m0(ws)
    xq, sfa = ops.quant_mxf8_act(x)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ops.cuda_ext().gemm_mxf8(y, xq, sfa, wq, wsf, None, None, 0, bn, ks)
    xs = ref.unpack_act_scales_ue8m0(sfa.cpu(), M, K)
    r = ref.fp8_block_gemm(xq.cpu(), xs, wq.cpu(), ws.cpu())
    rel = ((y.float().cpu() - r).norm() / r.norm()).item()
    assert rel < 1e-2, rel
    assert int(ops.cuda_ext().status()[0]) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("bn,ks", [(128, 1), (256, 1), (128, 4)])
def test_gemm_mxf8_silu_bias_residual(bn, ks):
    torch.manual_seed(11)
    M, I, K = 150, 1024, 2048
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wi = ops.interleave_gate_up(torch.randn(2 * I, K, device="cuda", dtype=torch.bfloat16) * 0.02)
    wq, ws = ref.quant_mxf8_weight(wi)
    wsf = ref.pack_block_scales_ue8m0(ws)
    xq, sfa = ops.quant_mxf8_act(x)
    xs = ref.unpack_act_scales_ue8m0(sfa.cpu(), M, K)
    out = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    ops.cuda_ext().gemm_mxf8(out, xq, sfa, wq, wsf, None, None, 1, bn, ks)
    full = ref.fp8_block_gemm(xq.cpu(), xs, wq.cpu(), ws.cpu()).view(M, I // 64, 2, 64)
    r = (torch.nn.functional.silu(full[:, :, 0]) * full[:, :, 1]).reshape(M, I)
    assert ((out.float().cpu() - r).norm() / r.norm()).item() < 1e-2
    y = torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    res = torch.randn(M, 2 * I, device="cuda", dtype=torch.bfloat16)
    bias = torch.randn(2 * I, device="cuda", dtype=torch.bfloat16)
    ops.cuda_ext().gemm_mxf8(y, xq, sfa, wq, wsf, bias, res, 0, bn, ks)
    r2 = ref.fp8_block_gemm(xq.cpu(), xs, wq.cpu(), ws.cpu()) + res.float().cpu() + bias.float().cpu()
    assert ((y.float().cpu() - r2).norm() / r2.norm()).item() < 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("M,H,add", [(1, 4096, False), (300, 4096, True), (129, 2048, True)])
def test_rms_norm_mxf8_matches_norm_then_quant(M, H, add):
    torch.manual_seed(M + H)
    x = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device="cuda")).to(torch.bfloat16)
    res = torch.randn(M, H, device="cuda", dtype=torch.bfloat16) if add else None
    res_ref = res.clone() if add else None
    xq, sfa = ops.rms_norm_mxf8(x, w, 1e-5, 0.0, residual=res)
    if add:
        y, res_ref = ops.fused_add_rms_norm(x, res_ref, w, 1e-5)
        assert torch.equal(res, res_ref)
    else:
        y = ops.rms_norm(x, w, 1e-5)
    qr, sr = ref.quant_mxf8_act(y.cpu())
    s = ref.unpack_act_scales_ue8m0(sfa.cpu(), M, H)
    deq = xq.float().cpu().view(M, H // 128, 128) * s.unsqueeze(-1)
    want = qr.float().view(M, H // 128, 128) * sr.unsqueeze(-1)
    # the fused kernel quantises the fp32 normalised values, the reference the bf16-rounded ones
    assert ((deq - want).norm() / want.norm()).item() < 2e-2
    assert (s == sr).float().mean().item() > 0.99


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 200, 1300])
def test_gemm_mxf8_silu_emits_mxf8_operand(M):
    torch.manual_seed(M)
    I, K = 1024, 2048
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    wi = ops.interleave_gate_up(torch.randn(2 * I, K, device="cuda", dtype=torch.bfloat16) * 0.02)
    wq, ws = ref.quant_mxf8_weight(wi)
    wsf = ref.pack_block_scales_ue8m0(ws)
    xq, sfa = ops.quant_mxf8_act(x)
    q, sf = ops.linear_mxf8_silu_q(xq, sfa, wq, wsf)
    bf = ops.linear_mxf8_q(xq, sfa, wq, wsf, silu_mul=True)            # same GEMM, bf16 epilogue
    qr, sr = ref.quant_mxf8_act(bf.cpu())
    s = ref.unpack_act_scales_ue8m0(sf.cpu(), M, I)
    deq = q.float().cpu().view(M, I // 128, 128) * s.unsqueeze(-1)
    want = qr.float().view(M, I // 128, 128) * sr.unsqueeze(-1)
    assert ((deq - want).norm() / want.norm()).item() < 2e-2
    assert int(ops.cuda_ext().status()[0]) == 0


_ORACLE = {}


def _llama3_oracle(mc, prompt):
    """fp32 CPU logits of the last prompt position on the unquantised random-init weights
    (the same seed every engine below starts from)."""
    key = (mc.num_hidden_layers, tuple(prompt))
    if key not in _ORACLE:
        from rusteeze_b200.models.loader import build_model, to_cpu_fp32
        from rusteeze_b200.models.naive import naive_logits
        m = build_model(mc, dtype=torch.bfloat16, device="cuda:0", seed=0)
        _ORACLE[key] = torch.log_softmax(naive_logits(to_cpu_fp32(m), prompt)[-1].double(), -1)
        del m
        torch.cuda.empty_cache()
    return _ORACLE[key]


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,tol", [("none", 0.08), ("ue8m0", 0.8), ("fp32", 0.7)])
def test_fp8_engine_logprobs_track_the_fp32_oracle(fmt, tol):
    """Llama-3-8B shapes (2 layers, random init): the first step's top-20 logprobs of the bf16
    engine, the MXFP8 engine (power-of-two UE8M0 block scales applied in the MMA) and the
    fp32-scale FP8 engine (per-K-block promotion) against the fp32 oracle on the unquantised
    weights.  The bound covers weight and activation quantisation together (measured on
    B200: 0.045 bf16, 0.60 MXFP8, 0.47 fp32-scale FP8, each with the oracle's top 5 in its
    top 20)."""
    from rusteeze_b200.config.config import Config, QuantizationConfig
    from rusteeze_b200.core.sampling_params import SamplingParams
    from rusteeze_b200.engine.llm_engine import LLMEngine
    from rusteeze_b200.models.config import get_preset
    mc = dataclasses.replace(get_preset("llama-3-8b"), num_hidden_layers=2)
    prompt = list(range(1000, 1100))
    ref_lsm = _llama3_oracle(mc, prompt)
    cfg = Config()
    cfg.model.device = "cuda:0"
    cfg.model.seed = 0
    if fmt != "none":
        cfg.model.quantization = QuantizationConfig(method="fp8_block", scale_format=fmt)
    cfg.engine.num_gpu_blocks = 64
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 256
    eng = LLMEngine(cfg, model_config=mc)
    eng.add_request("r", None, SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True, logprobs=20), prompt)
    out = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            out = o
    top = out.outputs[0].logprobs[0]
    err = max(abs(lp - float(ref_lsm[t])) for t, lp in top.items())
    # the oracle's own top 5 must appear among the engine's top 20
    ref_top5 = set(torch.topk(ref_lsm, 5).indices.tolist())
    overlap = len(ref_top5 & set(top))
    print(f"{fmt}: max |logprob - oracle| over the top 20 = {err:.4f}, oracle top-5 overlap {overlap}/5")
    assert err < tol, (fmt, err)
    assert overlap >= 4, (fmt, overlap)
