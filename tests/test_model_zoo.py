"""Model zoo: every architecture's paged, batched forward equals the naive
dense forward (CPU fp32 oracle), HF checkpoint round-trip, TP slicing."""
import dataclasses

import numpy as np
import pytest
import torch

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.core.types import ModelArchitecture as A
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig, tiny_variant
from rusteeze_b200.models.decoder import TPGroup
from rusteeze_b200.models.loader import build_model, save_hf_checkpoint
from rusteeze_b200.models.naive import naive_greedy, naive_logits

ARCHS = [A.LLAMA, A.MISTRAL, A.MIXTRAL, A.QWEN2, A.PHI3, A.GEMMA, A.GEMMA2]
# GPU oracle cases: every architecture, plus Llama with ALiBi instead of RoPE
GPU_CASES = [(a, {}) for a in ARCHS] + [(A.LLAMA, {"position_embedding": "alibi"})]


def _engine(mc, **kw):
    cfg = Config()
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 64
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 96
    cfg.engine.enable_chunked_prefill = True
    for k, v in kw.items():
        setattr(cfg.engine, k, v)
    return LLMEngine(cfg, model_config=mc)


@pytest.mark.parametrize("arch", ARCHS, ids=[a.value for a in ARCHS])
def test_arch_engine_matches_naive(arch):
    mc = tiny_variant(arch)
    eng = _engine(mc)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, mc.vocab_size, int(n)).tolist() for n in (40, 70, 9)]
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o.outputs[0].token_ids
    for rid, p in zip(ids, prompts):
        assert done[rid] == naive_greedy(eng.model, p, 10), arch


def test_alibi_slopes_follow_the_paper():
    from rusteeze_b200.ops import reference as ref
    s8 = ref.alibi_slopes(8)
    assert torch.allclose(s8, torch.tensor([2.0 ** -i for i in range(1, 9)]))
    s32 = ref.alibi_slopes(32)
    assert abs(float(s32[0]) - 2 ** -0.25) < 1e-7 and abs(float(s32[-1]) - 2 ** -8) < 1e-9
    # 12 heads: the 8 power-of-two slopes, then odd terms of the 16-head sequence
    s12 = ref.alibi_slopes(12)
    assert torch.allclose(s12[:8], s8)
    assert torch.allclose(s12[8:], torch.tensor([2.0 ** (-0.5 * k) for k in (1, 3, 5, 7)]))
    b = ref.alibi_bias(torch.tensor([0.5]), torch.arange(3, 5), torch.arange(5))
    assert b.shape == (1, 2, 5) and float(b[0, 1, 4]) == 0.0 and float(b[0, 0, 0]) == -1.5


@pytest.mark.parametrize("non_pow2", [False, True])
def test_alibi_engine_matches_naive(non_pow2):
    """ALiBi position encoding (no rotation, per-head linear logit bias) through the paged,
    chunked-prefill engine equals the dense oracle; 8 heads (or 6, a non-power of two)."""
    mc = tiny_variant(A.LLAMA, position_embedding="alibi", num_attention_heads=6 if non_pow2 else 8,
                      num_key_value_heads=2, head_dim=32)
    eng = _engine(mc)
    assert eng.model.alibi is not None and eng.model.alibi.numel() == mc.num_attention_heads
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, mc.vocab_size, int(n)).tolist() for n in (50, 130, 7)]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o.outputs[0].token_ids
    for rid, p in zip(ids, prompts):
        assert done[rid] == naive_greedy(eng.model, p, 8)
    # the bias matters: the same weights without it give other logits
    m = build_model(mc, dtype=torch.float32, seed=4)
    m_rope = build_model(dataclasses.replace(mc, position_embedding="rope"), dtype=torch.float32, seed=4)
    assert not torch.allclose(naive_logits(m, prompts[0])[-1], naive_logits(m_rope, prompts[0])[-1], atol=1e-3)


def test_alibi_config_roundtrip():
    mc = tiny_variant(A.LLAMA, position_embedding="alibi")
    d = mc.to_hf_dict()
    assert d["alibi"] is True
    assert ModelConfig.from_hf_dict(d).use_alibi
    assert not ModelConfig.from_hf_dict({k: v for k, v in d.items() if k != "alibi"}).use_alibi
    with pytest.raises(Exception):
        tiny_variant(A.LLAMA, position_embedding="learned")


def test_sliding_window_changes_output():
    mc = tiny_variant(A.MISTRAL, sliding_window=8)
    m = build_model(mc, dtype=torch.float32, seed=3)
    p = list(range(1, 40))
    full = naive_logits(build_model(dataclasses.replace(mc, sliding_window=None), dtype=torch.float32, seed=3), p)
    win = naive_logits(m, p)
    assert torch.allclose(full[:8], win[:8], atol=1e-5)     # first 8 positions see everything anyway
    assert not torch.allclose(full[-1], win[-1], atol=1e-4)


@pytest.mark.parametrize("arch", [A.LLAMA, A.MIXTRAL, A.QWEN2, A.GEMMA2])
def test_hf_checkpoint_roundtrip(tmp_path, arch):
    mc = tiny_variant(arch)
    m = build_model(mc, dtype=torch.float32, seed=5)
    save_hf_checkpoint(m, str(tmp_path), shard_bytes=200_000)     # forces several shards + index
    assert len(list(tmp_path.glob("*.safetensors"))) > 1
    mc2 = ModelConfig.from_json_file(str(tmp_path))
    assert mc2.architecture == arch and mc2.num_hidden_layers == mc.num_hidden_layers
    m2 = build_model(mc2, dtype=torch.float32, model_dir=str(tmp_path))
    p = [3, 1, 4, 1, 5, 9, 2, 6]
    assert torch.allclose(naive_logits(m, p), naive_logits(m2, p), atol=1e-5)


def test_pytorch_bin_checkpoint_loads(tmp_path):
    """The same weights saved as sharded pytorch_model-*.bin files (with index) load identically."""
    import json
    from safetensors.torch import load_file
    mc = tiny_variant(A.LLAMA)
    m = build_model(mc, dtype=torch.float32, seed=6)
    st = tmp_path / "st"
    save_hf_checkpoint(m, str(st), shard_bytes=200_000)
    out = tmp_path / "bin"
    out.mkdir()
    (out / "config.json").write_text((st / "config.json").read_text())
    wm = {}
    for j, f in enumerate(sorted(st.glob("*.safetensors"))):
        name = f"pytorch_model-{j + 1:05d}-of-00099.bin"
        tensors = load_file(str(f))
        torch.save(tensors, out / name)
        wm.update({k: name for k in tensors})
    (out / "pytorch_model.bin.index.json").write_text(json.dumps({"weight_map": wm}))
    m2 = build_model(ModelConfig.from_json_file(str(out)), dtype=torch.float32, model_dir=str(out))
    p = [7, 1, 8, 2, 8]
    assert torch.allclose(naive_logits(m, p), naive_logits(m2, p), atol=1e-5)


class _FakeTP(TPGroup):
    def __init__(self, rank, size):
        self.rank, self.size = rank, size


@pytest.mark.parametrize("tp", [2, 4])
def test_tp_slices_partition_full_weights(tp):
    mc = tiny_variant(A.LLAMA, num_attention_heads=8, num_key_value_heads=4, intermediate_size=256)
    full = build_model(mc, dtype=torch.float32, seed=11)
    shards = [build_model(mc, dtype=torch.float32, seed=11, tp=_FakeTP(r, tp)) for r in range(tp)]
    D, hq, hkv = mc.head_dim, mc.num_attention_heads // tp, mc.num_key_value_heads // tp
    for li in range(mc.num_hidden_layers):
        F = full.layers[li]
        q = torch.cat([s.layers[li].qkv[:hq * D] for s in shards])
        k = torch.cat([s.layers[li].qkv[hq * D:(hq + hkv) * D] for s in shards])
        v = torch.cat([s.layers[li].qkv[(hq + hkv) * D:] for s in shards])
        assert torch.equal(torch.cat([q, k, v]), F.qkv)
        assert torch.equal(torch.cat([s.layers[li].o for s in shards], dim=1), F.o)
        I = mc.intermediate_size // tp
        g = torch.cat([s.layers[li].gate_up[:I] for s in shards])
        u = torch.cat([s.layers[li].gate_up[I:] for s in shards])
        assert torch.equal(torch.cat([g, u]), F.gate_up)
        assert torch.equal(torch.cat([s.layers[li].down for s in shards], dim=1), F.down)
    emb = torch.cat([s.embed for s in shards])[:mc.vocab_size]
    assert torch.equal(emb, full.embed)


def test_model_config_parsing_variants():
    d = {"model_type": "qwen2", "hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 1,
         "num_attention_heads": 4, "num_key_value_heads": 2, "vocab_size": 100,
         "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                          "original_max_position_embeddings": 8192}, "eos_token_id": [5, 6]}
    mc = ModelConfig.from_hf_dict(d)
    assert mc.architecture == A.QWEN2 and mc.attention_bias and mc.eos_token_id == [5, 6]
    assert mc.rope_scaling.type == "llama3" and mc.head_dim == 16
    assert ModelConfig.from_hf_dict({**d, "model_type": "", "architectures": ["MixtralForCausalLM"],
                                     "num_local_experts": 8, "num_experts_per_tok": 2}).is_moe


@pytest.mark.gpu
@pytest.mark.parametrize("arch,extra", GPU_CASES, ids=[a.value + ("-alibi" if e else "") for a, e in GPU_CASES])
def test_arch_gpu_logprobs_match_fp32_oracle(arch, extra):
    """Every architecture on the sm_100a kernels (SwiGLU and Gemma's GeGLU in the GEMM's
    gated epilogue, MoE grouped GEMMs, biases, softcaps, windows): the first step's top-5
    logprobs against the dense fp32 CPU oracle on the same weights."""
    from rusteeze_b200.models.loader import to_cpu_fp32
    kw = dict(hidden_size=512, intermediate_size=1024, num_attention_heads=4, num_key_value_heads=2,
              head_dim=128, vocab_size=32000)
    if arch == A.GEMMA2:
        kw.update(query_pre_attn_scalar=128)
    kw.update(extra)
    mc = tiny_variant(arch, **kw)
    cfg = Config()
    cfg.model.device = "cuda:0"
    cfg.engine.num_gpu_blocks = 64
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 256
    eng = LLMEngine(cfg, model_config=mc)
    p = np.random.default_rng(3).integers(0, mc.vocab_size, 50).tolist()
    ref = torch.log_softmax(naive_logits(to_cpu_fp32(eng.model), p)[-1].double(), -1)
    eng.add_request("r", None, SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True, logprobs=5), p)
    out = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            out = o
    top = out.outputs[0].logprobs[0]
    err = max(abs(lp - float(ref[t])) for t, lp in top.items())
    assert err < 0.05, (arch, err)
