"""The allocation-free decode-attention entry point, called through its
exported C symbol, must match the regular entry point (caller-provided
workspace) on two calls in a row.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.  It also passes on its own in a
fresh process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 4 * 1024 * 1024
TOO_LARGE = -201


def _lib():
    import rusteeze_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    fn = lib.rz_decode_attention_noalloc
    i64, i32, vp, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float
    fn.argtypes = [vp, i64, vp, i64, vp, vp, i64, i32, vp, vp, i64, i32, i32, i32, i32, i32, f32, i32, f32, vp]
    fn.restype = ctypes.c_int
    st = lib.rz_decode_attention_noalloc_status
    st.argtypes = [vp]
    st.restype = ctypes.c_int
    return fn, st


def _inputs(seq_lens, Hq, Hkv, D, seed):
    g = torch.Generator().manual_seed(seed)
    S = len(seq_lens)
    max_blocks = max((n + 15) // 16 for n in seq_lens) + 1
    nb = sum((n + 15) // 16 for n in seq_lens) + 4
    cache = torch.randn(nb, 2, 2, Hkv, 16, D, generator=g).to(torch.bfloat16).cuda()
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(S, max_blocks, dtype=torch.int32)
    c = 0
    for i, n in enumerate(seq_lens):
        k = (n + 15) // 16
        bt[i, :k] = perm[c:c + k].int()
        c += k
    q = torch.randn(S, Hq, D, generator=g).to(torch.bfloat16).cuda()
    return cache, bt.cuda(), q, torch.tensor(seq_lens, dtype=torch.int32).cuda()


def _call(fn, out, q, kc, vc, sl, bt, Hkv, splits, scale):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.stride(0),
              kc.shape[0], sl.data_ptr(), bt.data_ptr(), bt.stride(0), q.shape[0], q.shape[1], Hkv, q.shape[2],
              splits, scale, 0, 0.0, stream)


@pytest.mark.parametrize("Hq,Hkv,D,splits", [(32, 8, 128, 6), (8, 8, 64, 3)])
def test_noalloc_matches_regular_entry_point_twice(Hq, Hkv, D, splits):
    from rusteeze_b200 import ops
    fn, status = _lib()
    seq_lens = [1, 17, 100, 513, 1040, 64, 300]
    cache, bt, q, sl = _inputs(seq_lens, Hq, Hkv, D, seed=Hq + D)
    kc, vc = cache[:, 1, 0], cache[:, 1, 1]
    scale = D ** -0.5
    # regular entry point with a caller-provided workspace
    ws = torch.empty(len(seq_lens) * Hq * splits * (D + 2), device="cuda")
    ref = torch.empty_like(q)
    ops.cuda_ext().decode_attention(ref, q, kc, vc, sl, bt, ws, len(seq_lens), scale, 0, 0.0, splits)
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _call(fn, out, q, kc, vc, sl, bt, Hkv, splits, scale) == 0
        torch.cuda.synchronize()
        a, b = out.float().cpu(), ref.float().cpu()
        assert torch.isfinite(a).all()
        assert ((a - b).norm() / b.norm()).item() < 1e-2
    assert status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0


def _compare_twice(fn, seq_lens, Hq, Hkv, D, splits, seed):
    from rusteeze_b200 import ops
    cache, bt, q, sl = _inputs(seq_lens, Hq, Hkv, D, seed=seed)
    kc, vc = cache[:, 1, 0], cache[:, 1, 1]
    scale = D ** -0.5
    ws = torch.empty(len(seq_lens) * Hq * splits * (D + 2), device=q.device)
    ref = torch.empty_like(q)
    ops.cuda_ext().decode_attention(ref, q, kc, vc, sl, bt, ws, len(seq_lens), scale, 0, 0.0, splits)
    torch.cuda.synchronize(q.device)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _call(fn, out, q, kc, vc, sl, bt, Hkv, splits, scale) == 0
        torch.cuda.synchronize(q.device)
        a, b = out.float().cpu(), ref.float().cpu()
        assert torch.isfinite(a).all()
        assert ((a - b).norm() / b.norm()).item() < 1e-2


def test_noalloc_largest_accepted_size():
    """16 sequences x 32 heads x 63 splits x (128 + 2) = 4,193,280 floats: the largest
    split count that fits for this shape (head_dim + 2 never divides the power-of-two
    array size, so no size ends exactly at its last float; this one ends 1,024 floats
    before it).  One more split is rejected."""
    fn, _ = _lib()
    Hq, Hkv, D, S = 32, 8, 128, 16
    splits = SCRATCH_FLOATS // (S * Hq * (D + 2))
    assert splits == 63 and S * Hq * splits * (D + 2) > SCRATCH_FLOATS - Hq * (D + 2)
    _compare_twice(fn, [1100 + 37 * i for i in range(S)], Hq, Hkv, D, splits, seed=7)
    cache, bt, q, sl = _inputs([64] * S, Hq, Hkv, D, seed=8)
    out = torch.empty_like(q)
    assert _call(fn, out, q, cache[:, 0, 0], cache[:, 0, 1], sl, bt, Hkv, splits + 1, 0.1) == TOO_LARGE


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_on_a_second_device_after_the_first():
    """The scratch address is looked up per device and kernels opt in to their shared
    memory per device, so a call on cuda:1 after calls on cuda:0 must work."""
    fn, status = _lib()
    _compare_twice(fn, [5, 200, 777], 32, 8, 128, 4, seed=11)
    with torch.cuda.device(1):
        _compare_twice(fn, [5, 200, 777, 1500], 32, 8, 128, 4, seed=12)
        assert status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0


def test_noalloc_rejects_sizes_beyond_scratch():
    fn, _ = _lib()
    Hq, Hkv, D = 32, 8, 128
    cache, bt, q, sl = _inputs([64] * 4, Hq, Hkv, D, seed=1)
    out = torch.empty_like(q)
    splits = SCRATCH_FLOATS // (4 * Hq * (D + 2)) + 1      # partials one split too many
    rc = _call(fn, out, q, cache[:, 0, 0], cache[:, 0, 1], sl, bt, Hkv, splits, 0.1)
    assert rc == TOO_LARGE
