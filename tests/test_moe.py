"""Mixture of experts: the fused router + top-k kernel, the grouped tcgen05
GEMM over 128-aligned expert segments, the whole MoE block vs the dense
per-expert fp32 oracle, and a Mixtral-shaped engine run (GPU).  CPU: the
dense-loop path of a tiny Mixtral matches the naive model."""
import dataclasses

import numpy as np
import pytest
import torch

from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref


def _moe_oracle(h, router, w13, w2, topk, e_lo=0, renorm=True):
    """fp32 dense oracle over local experts [e_lo, e_lo + w13.shape[0])."""
    hf = h.float().cpu()
    logits = hf @ router.float().cpu().t()
    p = torch.softmax(logits, -1)
    w, idx = p.topk(topk, -1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    out = torch.zeros_like(hf)
    for le in range(w13.shape[0]):
        rows, slot = (idx == e_lo + le).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        gu = hf[rows] @ w13[le].float().cpu().t()
        I = gu.shape[1] // 2
        a = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        y = a @ w2[le].float().cpu().t()
        out.index_add_(0, rows, y * w[rows, slot].unsqueeze(1))
    return out, w, idx


@pytest.mark.gpu
def test_moe_route_kernel_matches_oracle():
    torch.manual_seed(0)
    M, H, E, k = 333, 1024, 8, 2
    h = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    wr = (torch.randn(E, H, device="cuda") * 0.05).to(torch.bfloat16)
    tw = torch.empty(M, k, device="cuda")
    tid = torch.empty(M, k, device="cuda", dtype=torch.int32)
    cnt = torch.zeros(E, device="cuda", dtype=torch.int32)
    ops.cuda_ext().moe_route(tw, tid, cnt, h, wr, k, 0, E, True)
    logits = h.float() @ wr.float().t()
    w, idx = ref.moe_topk_softmax(logits, k)
    # compare where the top-k choice is not a near-tie
    p = torch.softmax(logits, -1).sort(-1, descending=True).values
    clear = (p[:, k - 1] - p[:, k]) > 1e-3
    assert torch.equal(tid.long()[clear].sort(-1).values, idx[clear].sort(-1).values)
    got_w = torch.gather(tw, 1, tid.long().argsort(-1))
    want_w = torch.gather(w, 1, idx.argsort(-1))
    assert torch.allclose(got_w[clear], want_w[clear], atol=1e-4)
    assert int(cnt.sum()) == M * k
    assert torch.equal(cnt.cpu(), torch.bincount(tid.long().flatten().cpu(), minlength=E).int())


@pytest.mark.gpu
@pytest.mark.parametrize("epi", [0, 1])
def test_grouped_gemm_matches_per_expert(epi):
    torch.manual_seed(1)
    G, N, K = 5, 1024, 512
    counts = [0, 130, 7, 256, 1]
    off, end, o = [], [], 0
    for c in counts:
        off.append(o)
        end.append(o + c)
        o += (c + 127) // 128 * 128
    off.append(o)
    x = torch.randn(o + 64, K, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(G, N, K, device="cuda") * 0.05).to(torch.bfloat16)
    wi = ops.interleave_gate_up_experts(w) if epi else w
    n_out = N // 2 if epi else N
    out = torch.zeros(o + 64, n_out, device="cuda", dtype=torch.bfloat16)
    go = torch.tensor(off, dtype=torch.int32, device="cuda")
    ge = torch.tensor(end, dtype=torch.int32, device="cuda")
    ops.cuda_ext().gemm_grouped(out, x, wi, go, ge, epi, 0)
    for g in range(G):
        if counts[g] == 0:
            continue
        r = x[off[g]:end[g]].float() @ w[g].float().t()
        if epi:
            r = torch.nn.functional.silu(r[:, :N // 2]) * r[:, N // 2:]
        got = out[off[g]:end[g]].float()
        assert ((got - r).norm() / r.norm()).item() < 1e-2, g
    # rows past a segment's end are never written
    assert out[end[1]:off[2]].abs().sum().item() == 0
    assert int(ops.cuda_ext().status()[0]) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("M,e_lo,ne", [(1, 0, 8), (37, 0, 8), (700, 0, 8), (300, 2, 2)])
def test_moe_block_matches_dense_oracle(M, e_lo, ne):
    torch.manual_seed(M + e_lo)
    H, I, E, k = 1024, 1792, 8, 2
    h = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    router = (torch.randn(E, H, device="cuda") * 0.05).to(torch.bfloat16)
    w13 = (torch.randn(ne, 2 * I, H, device="cuda") * 0.03).to(torch.bfloat16)
    w2 = (torch.randn(ne, H, I, device="cuda") * 0.03).to(torch.bfloat16)
    out = ops.moe_forward(h, router, ops.interleave_gate_up_experts(w13), w2, k, e_lo)
    want, _, _ = _moe_oracle(h, router, w13, w2, k, e_lo)
    rel = ((out.float().cpu() - want).norm() / want.norm().clamp_min(1e-6)).item()
    assert rel < 2e-2, rel


@pytest.mark.gpu
def test_mixtral_shaped_engine_runs_and_matches_oracle():
    from rusteeze_b200.config.config import Config
    from rusteeze_b200.core.sampling_params import SamplingParams
    from rusteeze_b200.engine.llm_engine import LLMEngine
    from rusteeze_b200.models.config import get_preset
    from rusteeze_b200.models.loader import to_cpu_fp32
    from rusteeze_b200.models.naive import naive_logits
    mc = dataclasses.replace(get_preset("mixtral-8x7b"), num_hidden_layers=2, hidden_size=1024,
                             intermediate_size=1792, num_attention_heads=8, num_key_value_heads=2)
    cfg = Config()
    cfg.model.device = "cuda:0"
    cfg.engine.num_gpu_blocks = 256
    cfg.engine.max_num_seqs = 8
    cfg.engine.max_num_batched_tokens = 1024
    eng = LLMEngine(cfg, model_config=mc)
    assert getattr(eng.model.layers[0], "w13_il", None) is not None
    rng = np.random.default_rng(0)
    p = rng.integers(0, mc.vocab_size, 120).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True, logprobs=5)
    eng.add_request("r", None, sp, p)
    out = None
    while eng.has_unfinished_requests():
        for o in eng.step():
            out = o
    lsm = torch.log_softmax(naive_logits(to_cpu_fp32(eng.model), p)[-1], -1)
    for tok, lp in out.outputs[0].logprobs[0].items():
        assert abs(lp - float(lsm[tok])) < 0.1
    # a batch of decodes through the CUDA graphs
    outs = []
    for i in range(6):
        eng.add_request(f"b{i}", None, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True),
                        rng.integers(0, mc.vocab_size, 40 + 17 * i).tolist())
    while eng.has_unfinished_requests():
        outs += [o for o in eng.step() if o.finished]
    assert len(outs) == 6 and all(len(o.outputs[0].token_ids) == 12 for o in outs)
    assert int(ops.cuda_ext().status()[0]) == 0
