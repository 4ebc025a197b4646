"""Speculative decoding: greedy output must equal plain greedy decoding
exactly, whatever the draft; a self-draft accepts everything."""
import numpy as np

from rusteeze_b200.config.config import Config, SpeculativeSection
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig

MC = ModelConfig(name="spec-tiny", hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2, vocab_size=512, max_position_embeddings=512)


def _engine(spec=None, device="cpu"):
    cfg = Config()
    cfg.model.device = device
    cfg.model.dtype = "float32" if device == "cpu" else "bfloat16"
    cfg.engine.num_gpu_blocks = 128
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 256
    cfg.engine.enable_chunked_prefill = True
    cfg.engine.speculative = spec
    return LLMEngine(cfg, model_config=MC)


def _run(eng, prompts, n=12, temp=0.0):
    sp = SamplingParams(temperature=temp, max_tokens=n, ignore_eos=True, seed=3)
    ids = [eng.add_request(None, None, sp, p).request_id for p in prompts]
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o.outputs[0].token_ids
    return [done[i] for i in ids]


PROMPTS = [np.random.default_rng(i).integers(0, 512, n).tolist() for i, n in enumerate((20, 45, 7))]


def test_self_draft_greedy_accepts_all_and_matches():
    ref = _run(_engine(), PROMPTS)
    eng = _engine(SpeculativeSection(num_speculative_tokens=4))
    got = _run(eng, PROMPTS)
    assert got == ref
    assert eng.spec.acceptance_rate() == 1.0 and eng.spec.stats["rounds"] > 0


def test_independent_draft_greedy_matches_target():
    ref = _run(_engine(), PROMPTS)
    eng = _engine(SpeculativeSection(draft_preset=None, num_speculative_tokens=3))
    # an independent draft: same architecture, different random weights
    from rusteeze_b200.models.loader import build_model
    sd = eng.spec
    sd.self_draft = False
    sd.draft = build_model(MC, dtype=eng.model.dtype, device="cpu", seed=99)
    from rusteeze_b200.engine.model_runner import ModelRunner
    r = eng.runner
    sd.drunner = ModelRunner(sd.draft, num_gpu_blocks=r.num_gpu_blocks, num_cpu_blocks=0, max_num_seqs=4,
                             max_num_batched_tokens=256, max_model_len=eng.max_model_len, use_cuda_graph=False)
    got = _run(eng, PROMPTS)
    assert got == ref
    assert 0.0 <= sd.acceptance_rate() < 1.0


def test_sampled_speculation_runs():
    eng = _engine(SpeculativeSection(num_speculative_tokens=2))
    out = _run(eng, PROMPTS, temp=0.8)
    assert all(len(o) == 12 for o in out)
