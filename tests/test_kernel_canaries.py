"""Out-of-bounds write canaries for the sm_100a kernels (compute-sanitizer is not available
here).  Each kernel writes into a view of a larger buffer whose guard regions -- extra
rows before and after, extra columns past N, the tail of a workspace -- hold a sentinel
bit pattern; after the kernel every guard must be bit-identical and the result still
match the oracle."""
import pytest
import torch

from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_SENTINEL = 0x7FAA            # a NaN payload no kernel produces
F32_SENTINEL = 0x7FC0DEAD


def C():
    return ops.cuda_ext()


def rel_err(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _guarded(rows, cols, pad_rows=2, pad_cols=0):
    """A bf16 buffer of (rows + 2 * pad_rows, cols + pad_cols) filled with the sentinel, and
    the [rows, cols] view the kernel writes into (rows pad_rows.., columns 0..cols)."""
    big = torch.empty(rows + 2 * pad_rows, cols + pad_cols, device=DEV, dtype=torch.bfloat16)
    big.view(torch.int16).fill_(BF16_SENTINEL)
    return big, big[pad_rows:pad_rows + rows, :cols]


def _guards_intact(big, rows, cols, pad_rows=2):
    b = big.view(torch.int16)
    ok = (b[:pad_rows] == BF16_SENTINEL).all() & (b[pad_rows + rows:] == BF16_SENTINEL).all()
    if big.shape[1] > cols:
        ok &= (b[:, cols:] == BF16_SENTINEL).all()
    return bool(ok)


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    torch.cuda.synchronize()
    assert int(C().status()[0]) == 0


@pytest.mark.parametrize("bn,ks", [(64, 1), (128, 1), (256, 1), (128, 2), (256, 4)])
@pytest.mark.parametrize("M", [1, 77, 300])
def test_gemm_bf16_writes_only_its_output(bn, ks, M):
    torch.manual_seed(M + bn)
    N, K = 328, 1024                     # N not a multiple of the tile: ragged last column tile
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.02
    big, out = _guarded(M, N, pad_cols=40)
    C().gemm_bf16_ex(out, x, w, None, None, 0, bn, ks)
    torch.cuda.synchronize()
    assert _guards_intact(big, M, N)
    assert rel_err(out, x.float() @ w.float().t()) < 1e-2


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("M", [5, 200])
def test_gemm_mxf8_writes_only_its_output(bn, M):
    torch.manual_seed(M + bn + 1)
    N, K = 384, 1024
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    wq, ws = ref.quant_mxf8_weight(torch.randn(N, K, device=DEV) * 0.02)
    xq, sfa = ops.quant_mxf8_act(x)
    big, out = _guarded(M, N, pad_cols=64)
    C().gemm_mxf8(out, xq, sfa, wq, ref.pack_block_scales_ue8m0(ws), None, None, 0, bn, 1)
    torch.cuda.synchronize()
    assert _guards_intact(big, M, N)
    xs = ref.unpack_act_scales_ue8m0(sfa, M, K)
    x_deq = (xq.float().view(M, K // 128, 128) * xs.unsqueeze(-1)).view(M, K)
    w_deq = (wq.float().view(N // 128, 128, K // 128, 128) * ws[:, None, :, None]).view(N, K)
    assert rel_err(out, x_deq @ w_deq.t()) < 1e-2


def _paged(seq_lens, q_lens, Hq, Hkv, D, seed):
    g = torch.Generator().manual_seed(seed)
    S = len(seq_lens)
    max_blocks = max((s + 15) // 16 for s in seq_lens) + 1
    nb = sum((s + 15) // 16 for s in seq_lens) + 8
    cache = torch.randn(nb, 2, Hkv, 16, D, generator=g).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(S, max_blocks, dtype=torch.int32)
    c = 0
    for i, s in enumerate(seq_lens):
        n = (s + 15) // 16
        bt[i, :n] = perm[c:c + n].int()
        c += n
    q = torch.randn(sum(q_lens), Hq, D, generator=g).to(torch.bfloat16)
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    return cache, bt, q, qsl, torch.tensor(seq_lens, dtype=torch.int32)


@pytest.mark.parametrize("splits", [1, 4])
def test_decode_attention_writes_only_its_output_and_workspace(splits):
    Hq, Hkv, D = 32, 8, 128
    seq_lens = [1, 17, 300, 1030]
    cache, bt, q, qsl, sl = _paged(seq_lens, [1] * 4, Hq, Hkv, D, seed=3)
    r = ref.paged_attention(q, cache[:, 0], cache[:, 1], qsl, sl, bt, D ** -0.5)
    cd = cache.to(DEV)
    need = len(seq_lens) * Hq * splits * (D + 2)
    ws_big = torch.empty(need + 4096, device=DEV)
    ws_big.view(torch.int32).fill_(F32_SENTINEL)
    big, out2d = _guarded(len(seq_lens), Hq * D)
    out = out2d.view(len(seq_lens), Hq, D)
    C().decode_attention(out, q.to(DEV), cd[:, 0], cd[:, 1], sl.to(DEV), bt.to(DEV), ws_big[:need], len(seq_lens),
                         D ** -0.5, 0, 0.0, splits)
    torch.cuda.synchronize()
    assert _guards_intact(big, len(seq_lens), Hq * D)
    assert bool((ws_big.view(torch.int32)[need:] == F32_SENTINEL).all())
    assert rel_err(out, r) < 1e-2


@pytest.mark.parametrize("impl", [1, 2])
def test_prefill_attention_writes_only_its_output(impl):
    Hq, Hkv, D = 32, 8, 128
    specs = [(77, 77), (300, 100), (130, 1), (129, 129)]
    cache, bt, q, qsl, sl = _paged([s for s, _ in specs], [x for _, x in specs], Hq, Hkv, D, seed=5)
    r = ref.paged_attention(q, cache[:, 0], cache[:, 1], qsl, sl, bt, D ** -0.5)
    cd = cache.to(DEV)
    T = q.shape[0]
    big, out2d = _guarded(T, Hq * D)
    out = out2d.view(T, Hq, D)
    C().prefill_attention_impl(out, q.to(DEV), cd[:, 0], cd[:, 1], qsl.to(DEV), sl.to(DEV), bt.to(DEV), 0,
                               len(specs), max(x for _, x in specs), D ** -0.5, 0, 0.0, impl)
    torch.cuda.synchronize()
    assert _guards_intact(big, T, Hq * D)
    assert rel_err(out, r) < 1.5e-2


def test_rope_and_cache_writes_only_the_mapped_slots():
    Hq, Hkv, D, T, nb = 32, 8, 128, 37, 16
    torch.manual_seed(9)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 500, (T,), device=DEV)
    cs = ref.rope_cos_sin_cache(D, 1024, 500000.0, device=DEV)
    cache = torch.empty(nb, 2, Hkv, 16, D, device=DEV, dtype=torch.bfloat16)
    cache.view(torch.int16).fill_(BF16_SENTINEL)
    slots = torch.randperm(nb * 16, device=DEV)[:T]
    ops.rope_and_cache(qkv, pos, cs, cache[:, 0], cache[:, 1], slots, Hq, Hkv, D)
    torch.cuda.synchronize()
    written = torch.zeros(nb * 16, dtype=torch.bool, device=DEV)
    written[slots] = True
    # [blocks, 2, Hkv, 16, D] -> per (k|v, head, slot): the untouched slots keep the sentinel
    per_slot = cache.view(torch.int16).permute(1, 2, 0, 3, 4).reshape(2, Hkv, nb * 16, D)
    assert bool((per_slot[:, :, ~written] == BF16_SENTINEL).all())
    assert not bool((per_slot[:, :, written] == BF16_SENTINEL).all())
