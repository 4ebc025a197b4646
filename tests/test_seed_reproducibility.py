"""Per-request seeds (CPU): a sampled request with a fixed seed emits the same tokens
whether it runs alone or batched with other traffic, under the synchronous and the
pipelined schedule, and with prefix caching on."""
import numpy as np
import pytest

from rusteeze_b200.config.config import Config
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.llm_engine import LLMEngine
from rusteeze_b200.models.config import ModelConfig

MC = ModelConfig(name="seeds", hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=2,
                 num_key_value_heads=1, vocab_size=300, max_position_embeddings=512)


def _engine(prefix=False, pipelined=False):
    cfg = Config()
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.engine.num_gpu_blocks = 128
    cfg.engine.max_num_seqs = 8
    cfg.engine.max_num_batched_tokens = 256
    cfg.engine.enable_prefix_caching = prefix
    eng = LLMEngine(cfg, model_config=MC)
    eng._async = pipelined
    return eng


def _run(eng, reqs):
    for rid, toks, sp in reqs:
        eng.add_request(rid, None, sp, toks)
    done = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                done[o.request_id] = o.outputs[0].token_ids
    return done


@pytest.mark.parametrize("prefix,pipelined", [(False, False), (True, False), (False, True)])
def test_seeded_request_is_reproducible_alone_and_batched(prefix, pipelined):
    rng = np.random.default_rng(0)
    target = ("target", rng.integers(0, 300, 30).tolist(),
              SamplingParams(temperature=0.9, top_p=0.95, top_k=50, max_tokens=20, seed=1234, ignore_eos=True))
    others = [(f"o{i}", rng.integers(0, 300, int(rng.integers(5, 60))).tolist(),
               SamplingParams(temperature=1.0, max_tokens=int(rng.integers(5, 25)), ignore_eos=True))
              for i in range(6)]
    alone = _run(_engine(prefix, pipelined), [target])["target"]
    batched = _run(_engine(prefix, pipelined), others[:3] + [target] + others[3:])["target"]
    assert len(alone) == 20 and alone == batched
