"""Tail split of the tcgen05 GEMM: when the last wave of tiles is thin, its tiles run as
K ranges on the otherwise idle SMs and the last-arriving split sums the partials.

CPU: the plan (split count, no empty K range, every tail tile's K covered exactly once,
one split unit per CTA at most).  GPU (opt-in with RZ_GEMM_TAIL_SPLIT=1, in a child
process since the switch is read once): bf16 and MXFP8 GEMMs at thin-last-wave shapes
against a plain fp32 reference, bit-identical across runs."""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _C():
    from rusteeze_b200 import ops
    return ops.cuda_ext()


def _units(S, full, tails, k_blocks):
    """Python restatement of the kernel's unit -> (tile, K range) mapping for tail units."""
    per = -(-k_blocks // S)
    out = []
    for v in range(tails * S):
        tail, ks = divmod(v, S)
        out.append((full + tail, ks * per, min(k_blocks, ks * per + per)))
    return out


@pytest.mark.parametrize("M,N,k_blocks,bn", [(1256, 4096, 112, 256), (1256, 4096, 32, 256), (1256, 6144, 32, 256),
                                             (300, 8192, 64, 128), (2000, 4096, 7, 256)])
def test_tail_plan_covers_k_exactly(M, N, k_blocks, bn):
    S, full, tails = _C().gemm_tail_plan(M, N, k_blocks, bn, 148)
    tiles = -(-M // 128) * -(-N // bn)
    if S <= 1:
        assert tiles <= 148 or tiles % 148 == 0 or 2 * (tiles % 148) > 148 or k_blocks < 2
        return
    assert tails == tiles % 148 and full == tiles - tails and full % 148 == 0
    assert tails * S <= 148                         # each CTA runs at most one split unit
    units = _units(S, full, tails, k_blocks)
    for t in range(full, tiles):
        ranges = sorted((a, b) for tt, a, b in units if tt == t)
        assert all(b > a for a, b in ranges)        # no empty split
        assert ranges[0][0] == 0 and ranges[-1][1] == k_blocks
        assert all(ranges[i][1] == ranges[i + 1][0] for i in range(len(ranges) - 1))


def test_tail_plan_examples():
    # Llama-3-8B o_proj / down at ~1256 tokens: 160 BN=256 tiles on 148 SMs -> 12 tail tiles
    assert _C().gemm_tail_plan(1256, 4096, 32, 256, 148) == [11, 148, 12]
    assert _C().gemm_tail_plan(1256, 4096, 112, 256, 148)[0] == 12
    assert _C().gemm_tail_plan(1000, 4096, 32, 256, 148)[0] <= 1     # 128 tiles: one wave


_CHILD = r"""
import torch
from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref
C = ops.cuda_ext()
torch.manual_seed(0)
worst = 0.0
for (M, N, K) in [(1256, 4096, 2048), (1256, 6144, 4096), (300, 8192, 1024)]:
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    want = x.float() @ w.float().t()
    for bn in (256, 128):
        outs = []
        for _ in range(2):
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            C.gemm_bf16_ex(out, x, w, None, None, 0, bn, 1)
            outs.append(out)
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1]), "tail split not reproducible"
        worst = max(worst, ((outs[0].float() - want).norm() / want.norm()).item())
    xq, sfa = ops.quant_mxf8_act(x)
    wq, ws = ref.quant_mxf8_weight(w)
    wsf = ref.pack_block_scales_ue8m0(ws)
    xs = ref.unpack_act_scales_ue8m0(sfa, M, K)
    x_deq = (xq.float().view(M, K // 128, 128) * xs.unsqueeze(-1)).view(M, K)
    w_deq = (wq.float().view(N // 128, 128, K // 128, 128) * ws[:, None, :, None]).view(N, K)
    want_q = x_deq @ w_deq.t()
    for bn in (256, 128):
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        C.gemm_mxf8(out, xq, sfa, wq, wsf, None, None, 0, bn, 1)
        torch.cuda.synchronize()
        worst = max(worst, ((out.float() - want_q).norm() / want_q.norm()).item())
assert int(C.status()[0]) == 0
print("TAIL_OK", worst)
"""


@pytest.mark.gpu
@pytest.mark.skipif(os.environ.get("RZ_GEMM_TAIL_SPLIT", "0") != "1", reason="tail split is opt-in (RZ_GEMM_TAIL_SPLIT=1)")
@pytest.mark.timeout(300)
def test_tail_split_gemm_matches_reference_on_gpu():
    r = subprocess.run([sys.executable, "-c", _CHILD], cwd=ROOT, capture_output=True, text=True, timeout=280,
                       env=dict(os.environ, RZ_GEMM_TAIL_SPLIT="1"))
    assert r.returncode == 0, r.stderr[-3000:]
    worst = float(r.stdout.split("TAIL_OK")[1])
    assert worst < 1e-2, worst
