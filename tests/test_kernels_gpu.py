"""sm_100a kernel numerics vs the fp32 PyTorch oracles (ops.reference)."""

import pytest
import torch

from rusteeze_b200 import ops
from rusteeze_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def C():
    return ops.cuda_ext()


def rel_err(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    torch.cuda.synchronize()
    st = C().status()
    assert int(st[0]) == 0, f"kernel status word set: {st.tolist()}"


# ----------------------------------------------------------------------------- norms / rope / act
@pytest.mark.parametrize("rows,H", [(1, 256), (7, 4096), (300, 4096), (33, 8192), (5, 2048)])
def test_rms_norm(rows, H):
    torch.manual_seed(0)
    x = torch.randn(rows, H, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(H, device=DEV, dtype=torch.bfloat16)
    y = ops.rms_norm(x, w, 1e-5)
    assert rel_err(y, ref.rms_norm(x.cpu(), w.cpu(), 1e-5)) < 1e-2
    r = torch.randn(rows, H, device=DEV, dtype=torch.bfloat16)
    r_ref = r.clone().cpu()
    y2, r2 = ops.fused_add_rms_norm(x, r, w, 1e-5, 1.0)
    yr, rr = ref.fused_add_rms_norm(x.cpu(), r_ref, w.cpu(), 1e-5, 1.0)
    assert rel_err(r2, rr) < 1e-2
    assert rel_err(y2, yr) < 1e-2


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (4, 1, 128), (8, 2, 64), (8, 4, 256)])
def test_rope_and_cache(Hq, Hkv, D):
    torch.manual_seed(1)
    T, nb = 37, 16
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 500, (T,), device=DEV)
    cs = ref.rope_cos_sin_cache(D, 1024, 500000.0, device=DEV)
    cache = torch.zeros(nb, 3, 2, Hkv, 16, D, device=DEV, dtype=torch.bfloat16)   # [blocks, L, 2, Hkv, 16, D]
    kc, vc = cache[:, 1, 0], cache[:, 1, 1]
    slots = torch.randperm(nb * 16, device=DEV)[:T]
    slots[3] = -1
    q_ref_in = qkv.clone().cpu()
    q = ops.rope_and_cache(qkv, pos, cs, kc, vc, slots, Hq, Hkv, D)
    kc_ref = torch.zeros(nb, Hkv, 16, D, dtype=torch.bfloat16)
    vc_ref = torch.zeros_like(kc_ref)
    q_ref = ops.rope_and_cache(q_ref_in, pos.cpu(), cs.cpu(), kc_ref, vc_ref, slots.cpu(), Hq, Hkv, D)
    assert rel_err(q, q_ref) < 1e-2
    assert rel_err(kc, kc_ref) < 1e-2
    assert torch.equal(vc.cpu(), vc_ref)
    assert cache[:, 0].abs().sum() == 0 and cache[:, 2].abs().sum() == 0   # other layers untouched


@pytest.mark.parametrize("kind", [0, 1])
def test_act_mul(kind):
    x = torch.randn(77, 2 * 1792, device=DEV, dtype=torch.bfloat16)
    y = ops.silu_mul(x) if kind == 0 else ops.gelu_tanh_mul(x)
    r = ref.silu_mul(x.cpu()) if kind == 0 else ref.gelu_tanh_mul(x.cpu())
    assert rel_err(y, r) < 1e-2


# ----------------------------------------------------------------------------- GEMM
SHAPES = [(1, 256, 256), (7, 4096, 4096), (128, 6144, 4096), (300, 4096, 4096), (1256, 1024, 4096),
          (129, 384, 1024), (64, 128256 // 8, 512), (2048, 2048, 2048), (40, 4096, 14336)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bf16_auto(M, N, K):
    torch.manual_seed(2)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.02
    y = ops.linear(x, w)
    r = x.float() @ w.float().t()
    assert rel_err(y, r) < 1e-2


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("ks", [1, 2, 4])
def test_gemm_bf16_tiles_splits(bn, ks):
    torch.manual_seed(3)
    M, N, K = 200, 768, 2048
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) * 0.02
    b = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    C().gemm_bf16_ex(out, x, w, b, res, 0, bn, ks)
    r = x.float() @ w.float().t() + b.float() + res.float()
    assert rel_err(out, r) < 1e-2


@pytest.mark.parametrize("bn,ks", [(128, 1), (256, 1), (128, 4), (256, 2)])
def test_gemm_silu_epilogue(bn, ks):
    torch.manual_seed(4)
    M, I, K = 150, 512, 1024
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    wg = torch.randn(I, K, device=DEV, dtype=torch.bfloat16) * 0.05
    wu = torch.randn(I, K, device=DEV, dtype=torch.bfloat16) * 0.05
    # interleave gate/up in 64-row blocks: [g0..63 | u0..63 | g64..127 | u64..127 | ...]
    wi = torch.stack([wg.view(I // 64, 64, K), wu.view(I // 64, 64, K)], dim=1).reshape(2 * I, K)
    out = torch.empty(M, I, device=DEV, dtype=torch.bfloat16)
    C().gemm_bf16_ex(out, x, wi, None, None, 1, bn, ks)
    g = x.float() @ wg.float().t()
    u = x.float() @ wu.float().t()
    r = torch.nn.functional.silu(g) * u
    assert rel_err(out, r) < 1.5e-2


def test_gemm_strided_activation():
    # q/k/v-style column slice of a wider activation buffer
    torch.manual_seed(5)
    big = torch.randn(96, 1024 + 256, device=DEV, dtype=torch.bfloat16)
    x = big[:, :1024]
    w = torch.randn(512, 1024, device=DEV, dtype=torch.bfloat16) * 0.03
    y = ops.linear(x, w)
    assert rel_err(y, x.float() @ w.float().t()) < 1e-2


# ----------------------------------------------------------------------------- attention
def _paged_setup(seq_lens, q_lens, Hq, Hkv, D, nb=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    S = len(seq_lens)
    max_blocks = max((l + 15) // 16 for l in seq_lens) + 1
    nb = nb or sum((l + 15) // 16 for l in seq_lens) + 8
    cache = torch.randn(nb, 2, 2, Hkv, 16, D, generator=g).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(S, max_blocks, dtype=torch.int32)
    c = 0
    for i, l in enumerate(seq_lens):
        n = (l + 15) // 16
        bt[i, :n] = perm[c:c + n].int()
        c += n
    T = sum(q_lens)
    q = torch.randn(T, Hq, D, generator=g).to(torch.bfloat16)
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    return cache, bt, q, qsl, torch.tensor(seq_lens, dtype=torch.int32)


class _Meta:
    pass


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (8, 8, 128), (4, 1, 128), (16, 2, 64), (8, 1, 128)])
@pytest.mark.parametrize("splits", [1, 3, 8])
def test_decode_attention(Hq, Hkv, D, splits):
    seq_lens = [1, 15, 16, 17, 100, 511, 1030, 64]
    cache, bt, q, qsl, sl = _paged_setup(seq_lens, [1] * len(seq_lens), Hq, Hkv, D)
    layer = 1
    kc, vc = cache[:, layer, 0], cache[:, layer, 1]
    r = ref.paged_attention(q, kc, vc, qsl, sl, bt, D ** -0.5)
    cache_d = cache.to(DEV)
    ws = torch.empty(len(seq_lens) * Hq * splits * (D + 2), device=DEV)
    out = torch.empty(q.shape, device=DEV, dtype=torch.bfloat16)
    C().decode_attention(out, q.to(DEV), cache_d[:, layer, 0], cache_d[:, layer, 1], sl.to(DEV), bt.to(DEV), ws,
                         len(seq_lens), D ** -0.5, 0, 0.0, splits)
    assert rel_err(out, r) < 1e-2


@pytest.mark.parametrize("window,softcap", [(0, 0.0), (37, 0.0), (0, 30.0)])
def test_decode_attention_window_softcap(window, softcap):
    Hq, Hkv, D = 8, 2, 128
    seq_lens = [5, 90, 300]
    cache, bt, q, qsl, sl = _paged_setup(seq_lens, [1] * 3, Hq, Hkv, D, seed=5)
    kc, vc = cache[:, 0, 0], cache[:, 0, 1]
    r = ref.paged_attention(q, kc, vc, qsl, sl, bt, D ** -0.5, window or None, softcap or None)
    cd = cache.to(DEV)
    ws = torch.empty(3 * Hq * 4 * (D + 2), device=DEV)
    out = torch.empty(q.shape, device=DEV, dtype=torch.bfloat16)
    C().decode_attention(out, q.to(DEV), cd[:, 0, 0], cd[:, 0, 1], sl.to(DEV), bt.to(DEV), ws, 3, D ** -0.5,
                         window, softcap, 4)
    assert rel_err(out, r) < 1e-2


def test_decode_attention_empty_rows_are_zero():
    Hq, Hkv, D = 8, 2, 128
    cache, bt, q, qsl, sl = _paged_setup([33, 20], [1, 1], Hq, Hkv, D)
    sl[1] = 0
    cd = cache.to(DEV)
    out = torch.full(q.shape, 7.0, device=DEV, dtype=torch.bfloat16)
    ws = torch.empty(2 * Hq * 2 * (D + 2), device=DEV)
    for splits in (1, 2):
        C().decode_attention(out, q.to(DEV), cd[:, 0, 0], cd[:, 0, 1], sl.to(DEV), bt.to(DEV), ws, 2, 0.1, 0, 0.0,
                             splits)
        assert out[1].abs().max().item() == 0.0


@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (4, 1, 128), (8, 4, 64), (8, 8, 256)])
def test_prefill_attention_varlen_chunked(Hq, Hkv, D):
    # (seq_len, q_len): full prompts, chunked continuations, 1-token tails
    specs = [(77, 77), (200, 64), (130, 1), (1000, 300), (16, 16), (65, 65)]
    seq_lens = [s for s, _ in specs]
    q_lens = [q for _, q in specs]
    cache, bt, q, qsl, sl = _paged_setup(seq_lens, q_lens, Hq, Hkv, D, seed=7)
    kc, vc = cache[:, 0, 0], cache[:, 0, 1]
    r = ref.paged_attention(q, kc, vc, qsl, sl, bt, D ** -0.5)
    cd = cache.to(DEV)
    out = torch.empty(q.shape, device=DEV, dtype=torch.bfloat16)
    C().prefill_attention(out, q.to(DEV), cd[:, 0, 0], cd[:, 0, 1], qsl.to(DEV), sl.to(DEV), bt.to(DEV), 0,
                          len(specs), max(q_lens), D ** -0.5, 0, 0.0)
    assert rel_err(out, r) < 1.5e-2


@pytest.mark.parametrize("window,softcap", [(40, 0.0), (0, 50.0)])
def test_prefill_attention_window_softcap(window, softcap):
    Hq, Hkv, D = 8, 2, 128
    specs = [(150, 150), (300, 100)]
    cache, bt, q, qsl, sl = _paged_setup([s for s, _ in specs], [x for _, x in specs], Hq, Hkv, D, seed=9)
    kc, vc = cache[:, 0, 0], cache[:, 0, 1]
    r = ref.paged_attention(q, kc, vc, qsl, sl, bt, D ** -0.5, window or None, softcap or None)
    cd = cache.to(DEV)
    out = torch.empty(q.shape, device=DEV, dtype=torch.bfloat16)
    C().prefill_attention(out, q.to(DEV), cd[:, 0, 0], cd[:, 0, 1], qsl.to(DEV), sl.to(DEV), bt.to(DEV), 0, 2,
                          150, D ** -0.5, window, softcap)
    assert rel_err(out, r) < 1.5e-2


# ----------------------------------------------------------------------------- sampling
def test_argmax_sample_exact():
    torch.manual_seed(11)
    logits = torch.randn(64, 128256, device=DEV)
    tok, lp = ops.sample(logits, None, None, None, None, None, None, greedy_all=True, want_logprobs=True)
    assert torch.equal(tok.cpu(), logits.argmax(-1).cpu())
    ref_lp = torch.log_softmax(logits, -1).gather(1, tok.view(-1, 1)).view(-1)
    assert torch.allclose(lp, ref_lp, atol=1e-3)


def _sample(logits, T, k, p, mp, seed, off):
    B = logits.shape[0]
    f = lambda v, dt: torch.full((B,), v, dtype=dt, device=DEV)  # noqa: E731
    return ops.sample(logits, f(T, torch.float32), f(k, torch.int32), f(p, torch.float32), f(mp, torch.float32),
                      torch.arange(B, device=DEV, dtype=torch.int64) + seed, f(off, torch.int64), greedy_all=False)


@pytest.mark.parametrize("T,k,p,mp", [(0.7, -1, 0.9, 0.0), (1.0, 50, 1.0, 0.0), (1.3, 20, 0.5, 0.0),
                                      (1.0, -1, 1.0, 0.05)])
def test_sampling_support_matches_reference(T, k, p, mp):
    torch.manual_seed(12)
    V = 32000
    logits = torch.randn(256, V, device=DEV) * 3
    tok, lp = _sample(logits, T, k, p, mp, 1, 0)
    probs = ref.topk_topp_minp_probs(logits.cpu(), torch.full((256,), T), torch.full((256,), k),
                                     torch.full((256,), p), torch.full((256,), mp))
    chosen = probs.gather(1, tok.cpu().view(-1, 1)).view(-1)
    assert (chosen > 0).all(), "sampled a token outside the filtered support"
    # the kernel reports the token's logprob under the temperature-scaled softmax of the whole row
    full = torch.log_softmax(logits.cpu() / T, -1).gather(1, tok.cpu().view(-1, 1)).view(-1)
    assert torch.allclose(lp.cpu(), full, atol=2e-3)


def test_sampling_distribution_chi_square():
    V = 16
    logits = torch.tensor([[3.0, 2.5, 2.0, 1.0, 0.5, 0.0] + [-1.0] * (V - 6)], device=DEV).repeat(4096, 1)
    T, p = 0.8, 0.9
    tok, _ = _sample(logits, T, -1, p, 0.0, 1000, 3)
    probs = ref.topk_topp_minp_probs(logits[:1].cpu(), torch.tensor([T]), torch.tensor([-1]), torch.tensor([p]),
                                     torch.tensor([0.0]))[0]
    cnt = torch.bincount(tok.cpu(), minlength=V).float()
    exp = probs * 4096
    keep = exp > 0
    assert (cnt[~keep] == 0).all()
    chi2 = (((cnt - exp) ** 2)[keep] / exp[keep]).sum().item()
    assert chi2 < 30.0, chi2   # dof <= 5


def test_sampling_seed_determinism():
    logits = torch.randn(32, 5000, device=DEV)
    a, _ = _sample(logits, 1.0, -1, 0.95, 0.0, 7, 11)
    b, _ = _sample(logits, 1.0, -1, 0.95, 0.0, 7, 11)
    c, _ = _sample(logits, 1.0, -1, 0.95, 0.0, 7, 12)
    assert torch.equal(a, b) and not torch.equal(a, c)


def test_spec_verify_greedy():
    B, k, V = 5, 4, 1000
    target = torch.randn(B * (k + 1), V, device=DEV)
    am = target.argmax(-1).view(B, k + 1)
    draft = am[:, :k].clone()
    draft[1, 0] = (draft[1, 0] + 1) % V
    draft[2, 2] = (draft[2, 2] + 1) % V
    out = torch.empty(B, k + 1, dtype=torch.int64, device=DEV)
    n = torch.empty(B, dtype=torch.int32, device=DEV)
    z = torch.zeros(B, device=DEV)
    C().spec_verify(out, n, target, None, draft, z, torch.zeros(B, dtype=torch.int64, device=DEV),
                    torch.zeros(B, dtype=torch.int64, device=DEV))
    acc_ref, out_ref = ref.spec_verify_greedy(draft.cpu(), am.cpu())
    assert torch.equal(n.cpu().long(), acc_ref)
    assert torch.equal(out.cpu(), out_ref)


def test_spec_verify_sampled_is_distribution_preserving():
    # draft q and target p over 6 tokens; the emitted first token must follow p
    V, N = 6, 20000
    p = torch.tensor([0.4, 0.3, 0.1, 0.1, 0.05, 0.05])
    q = torch.tensor([0.1, 0.1, 0.5, 0.1, 0.1, 0.1])
    tl = p.log().repeat(N * 2, 1).to(DEV)       # rows j=0 and j=1 (bonus) per sequence, k=1
    dl = q.log().repeat(N, 1).to(DEV)
    g = torch.Generator().manual_seed(0)
    draft = torch.multinomial(q, N, replacement=True, generator=g).view(N, 1).to(DEV)
    out = torch.empty(N, 2, dtype=torch.int64, device=DEV)
    n = torch.empty(N, dtype=torch.int32, device=DEV)
    C().spec_verify(out, n, tl, dl, draft, torch.ones(N, device=DEV), torch.arange(N, device=DEV),
                    torch.zeros(N, dtype=torch.int64, device=DEV))
    first = out[:, 0].cpu()
    freq = torch.bincount(first, minlength=V).float() / N
    assert (freq - p).abs().max() < 0.02


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (8, 8), (16, 2)])
@pytest.mark.parametrize("window,softcap", [(0, 0.0), (100, 0.0), (0, 30.0)])
def test_prefill_tcgen05_matches_mma_sync_and_oracle(Hq, Hkv, window, softcap):
    """tcgen05 FlashAttention prefill (impl 2) vs the mma.sync kernel (impl 1) and the fp32 oracle,
    over full prompts, chunked continuations (context > 0), 1-token tails and long sequences."""
    D = 128
    specs = [(77, 77), (300, 100), (130, 1), (2048, 700), (16, 16), (129, 129), (1000, 1000)]
    seq_lens = [s for s, _ in specs]
    q_lens = [q for _, q in specs]
    cache, bt, q, qsl, sl = _paged_setup(seq_lens, q_lens, Hq, Hkv, D, seed=21)
    kc, vc = cache[:, 0, 0], cache[:, 0, 1]
    r = ref.paged_attention(q, kc, vc, qsl, sl, bt, D ** -0.5, window or None, softcap or None)
    cd = cache.to(DEV)
    outs = []
    for impl in (1, 2):
        out = torch.zeros(q.shape, device=DEV, dtype=torch.bfloat16)
        C().prefill_attention_impl(out, q.to(DEV), cd[:, 0, 0], cd[:, 0, 1], qsl.to(DEV), sl.to(DEV), bt.to(DEV),
                                   0, len(specs), max(q_lens), D ** -0.5, window, softcap, impl)
        outs.append(out)
    assert rel_err(outs[1], r) < 1.5e-2
    assert rel_err(outs[1], outs[0].float()) < 1.5e-2
    assert int(C().status()[0]) == 0


@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (32, 8), (12, 4)])
@pytest.mark.parametrize("window", [0, 60])
def test_attention_alibi_matches_oracle(Hq, Hkv, window):
    """ALiBi slopes (power-of-two and interleaved non-power-of-two head counts) in the decode
    kernel (1 and 4 splits), the mma.sync prefill kernel and the tcgen05 prefill kernel (where
    the query heads per kv head divide 128) against the fp32 oracle."""
    D = 128
    slopes = ref.alibi_slopes(Hq)
    specs = [(77, 77), (300, 100), (130, 1), (700, 700), (16, 16)]
    cache, bt, q, qsl, sl = _paged_setup([s for s, _ in specs], [x for _, x in specs], Hq, Hkv, D, seed=31)
    kc, vc = cache[:, 0, 0], cache[:, 0, 1]
    r = ref.paged_attention(q, kc, vc, qsl, sl, bt, D ** -0.5, window or None, None, slopes)
    cd = cache.to(DEV)
    al = slopes.to(DEV)
    for impl in (1, 0):
        out = torch.zeros(q.shape, device=DEV, dtype=torch.bfloat16)
        C().prefill_attention_impl(out, q.to(DEV), cd[:, 0, 0], cd[:, 0, 1], qsl.to(DEV), sl.to(DEV), bt.to(DEV),
                                   0, len(specs), max(x for _, x in specs), D ** -0.5, window, 0.0, impl, al)
        assert rel_err(out, r) < 1.5e-2, impl
    # decode: one query row per sequence (the last position)
    dq_rows = [int(qsl[i + 1]) - 1 for i in range(len(specs))]
    dq = q[dq_rows].contiguous()
    dqsl = torch.arange(len(specs) + 1, dtype=torch.int32)
    rd = ref.paged_attention(dq, kc, vc, dqsl, sl, bt, D ** -0.5, window or None, None, slopes)
    for splits in (1, 4):
        ws = torch.empty(len(specs) * Hq * splits * (D + 2), device=DEV)
        out = torch.zeros(dq.shape, device=DEV, dtype=torch.bfloat16)
        C().decode_attention(out, dq.to(DEV), cd[:, 0, 0], cd[:, 0, 1], sl.to(DEV), bt.to(DEV), ws, len(specs),
                             D ** -0.5, window, 0.0, splits, al)
        assert rel_err(out, rd) < 1e-2, splits
    assert int(C().status()[0]) == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_kernels_on_a_second_device_after_the_first():
    """Kernels that opt in to more than 48 KB of shared memory do so per device: one process
    that launches on cuda:0 and then on cuda:1 (data-parallel replicas on threads) must get
    correct results on both."""
    D, Hq, Hkv = 128, 32, 8
    specs = [(300, 300), (700, 1), (90, 1)]
    cache, bt, q, qsl, sl = _paged_setup([s for s, _ in specs], [x for _, x in specs], Hq, Hkv, D, seed=31)
    r_pf = ref.paged_attention(q, cache[:, 0, 0], cache[:, 0, 1], qsl, sl, bt, D ** -0.5)
    dq, dsl = q[300:], sl[1:]
    r_dec = ref.paged_attention(dq, cache[:, 0, 0], cache[:, 0, 1], torch.arange(3, dtype=torch.int32), dsl,
                                bt[1:], D ** -0.5)
    torch.manual_seed(3)
    x = torch.randn(300, 4096, dtype=torch.bfloat16)
    w = torch.randn(1024, 4096, dtype=torch.bfloat16) * 0.02
    r_mm = x.float() @ w.float().t()
    for dev in ("cuda:0", "cuda:1"):
        with torch.cuda.device(dev):
            cd = cache.to(dev)
            out = torch.zeros(q.shape, device=dev, dtype=torch.bfloat16)
            C().prefill_attention(out, q.to(dev), cd[:, 0, 0], cd[:, 0, 1], qsl.to(dev), sl.to(dev), bt.to(dev), 0,
                                  1, 300, D ** -0.5, 0, 0.0)
            ws = torch.empty(2 * Hq * 4 * (D + 2), device=dev)
            dout = torch.empty(dq.shape, device=dev, dtype=torch.bfloat16)
            C().decode_attention(dout, dq.to(dev), cd[:, 0, 0], cd[:, 0, 1], dsl.to(dev), bt[1:].to(dev), ws, 2,
                                 D ** -0.5, 0, 0.0, 4)
            y = ops.linear(x.to(dev), w.to(dev))
            torch.cuda.synchronize(dev)
            assert rel_err(out[:300], r_pf[:300]) < 1.5e-2
            assert rel_err(dout, r_dec) < 1e-2
            assert rel_err(y, r_mm) < 1e-2
            assert int(C().status()[0]) == 0


def test_bounded_peer_wait_reports_timeout_and_context_survives():
    """Failure detection on the device without a fault: the fused TP boundary
    kernel waits for reduce-scatter flags that nothing sets (two 'ranks' whose
    peer buffers are local tensors).  The wait gives up after ~1 s, the status
    word reports kCommPeerTimeout (4) and the CUDA context keeps working."""
    import time
    H, rs_rows, M = 1024, 8, 16
    slots = torch.zeros(2 * rs_rows * H, device=DEV, dtype=torch.bfloat16)
    rs_flag = torch.zeros(4096, device=DEV, dtype=torch.int32)
    gathers = [torch.zeros(M + 128, H, device=DEV, dtype=torch.bfloat16) for _ in range(2)]
    ag = [torch.zeros(64, device=DEV, dtype=torch.int32) for _ in range(2)]
    residual = torch.zeros(rs_rows, H, device=DEV, dtype=torch.bfloat16)
    w = torch.ones(H, device=DEV, dtype=torch.bfloat16)
    epoch = torch.zeros(1, device=DEV, dtype=torch.int32)
    C().status().zero_()
    torch.cuda.synchronize()
    t0 = time.monotonic()
    C().rs_norm_ag(slots, rs_flag, 1, None, residual, w, 1e-5, 0.0, [g.data_ptr() for g in gathers],
                   [a.data_ptr() for a in ag], 0, M, rs_rows, epoch, 1, 0, None)
    torch.cuda.synchronize()
    dt = time.monotonic() - t0
    assert int(C().status()[0]) == 4
    assert 0.5 < dt < 30.0
    C().status().zero_()
    x = torch.randn(64, 64, device=DEV)
    assert torch.allclose((x @ x.t()).cpu(), x.cpu() @ x.cpu().t(), atol=1e-3)


# ----------------------------------------------------------------------------- embedding / LayerNorm / GeGLU
def test_embedding_vocab_shard_and_scale():
    torch.manual_seed(21)
    V, H, lo, rows = 1000, 512, 300, 250
    full = torch.randn(V, H, dtype=torch.bfloat16)
    ids = torch.randint(0, V, (77,))
    out = ops.embedding(ids.to(DEV), full[lo:lo + rows].to(DEV), lo, V, 7.5)
    own = (ids >= lo) & (ids < lo + rows)
    want = full.float()[ids] * 7.5 * own.unsqueeze(1).float()
    assert rel_err(out, want) < 5e-3
    assert (out.float().cpu()[~own] == 0).all()


@pytest.mark.parametrize("H,bias,res", [(512, True, False), (4096, False, True), (5120, True, True)])
def test_layer_norm(H, bias, res):
    torch.manual_seed(22)
    x = torch.randn(37, H, dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H)).to(torch.bfloat16)
    b = (0.1 * torch.randn(H)).to(torch.bfloat16) if bias else None
    r = torch.randn(37, H, dtype=torch.bfloat16) if res else None
    want_x = (x.float() + r.float()).to(torch.bfloat16) if res else x
    want = ref.layer_norm(want_x, w, b, 1e-5)
    rd = r.to(DEV) if res else None
    y = ops.layer_norm(x.to(DEV), w.to(DEV), b.to(DEV) if bias else None, 1e-5, residual=rd)
    assert rel_err(y, want) < 1e-2
    if res:
        assert torch.equal(rd.cpu(), want_x)


@pytest.mark.parametrize("M", [7, 300])
def test_gelu_gated_epilogue_bf16_and_mxfp8(M):
    """GELU(tanh)(gate) * up in the GEMM epilogue (Gemma's GeGLU), bf16 and MXFP8 (bf16
    output and the re-quantised MXFP8 operand) vs the fp32 oracle."""
    torch.manual_seed(23)
    K, I = 1024, 512
    x = torch.randn(M, K, dtype=torch.bfloat16, device=DEV)
    wg = (torch.randn(I, K) * 0.05).to(torch.bfloat16)
    wu = (torch.randn(I, K) * 0.05).to(torch.bfloat16)
    w_il = ops.interleave_gate_up(torch.cat([wg, wu]).to(DEV))
    g, u = x.float() @ wg.to(DEV).float().t(), x.float() @ wu.to(DEV).float().t()
    want = torch.nn.functional.gelu(g, approximate="tanh") * u
    assert rel_err(ops.linear_silu_mul(x, w_il, act="gelu_tanh"), want) < 1.5e-2
    assert rel_err(ops.linear_silu_mul(x, w_il, act="silu"), torch.nn.functional.silu(g) * u) < 1.5e-2
    # MXFP8: weights and activations quantised, compare against the dequantised oracle
    q, s = ref.quant_mxf8_weight(w_il.float().cpu())
    wsf = ref.pack_block_scales_ue8m0(s).to(DEV)
    wdq = (q.float().view(-1, 128, K // 128, 128) * s[:, None, :, None]).view(2 * I, K)
    xq, sfa = ops.quant_mxf8_act(x)
    xr_q, xr_s = ref.quant_mxf8_act(x.cpu())
    xdq = (xr_q.float().view(M, K // 128, 128) * xr_s.unsqueeze(-1)).view(M, K)
    y = (xdq @ wdq.t()).view(M, I // 64, 2, 64)
    want_mx = (torch.nn.functional.gelu(y[:, :, 0], approximate="tanh") * y[:, :, 1]).reshape(M, I)
    out = ops.linear_mxf8_q(xq, sfa, q.to(DEV), wsf, silu_mul=True, act="gelu_tanh")
    assert rel_err(out, want_mx) < 2e-2
    oq, osf = ops.linear_mxf8_silu_q(xq, sfa, q.to(DEV), wsf, act="gelu_tanh")
    o_deq = (oq.float().cpu().view(M, I // 128, 128) * ref.unpack_act_scales_ue8m0(osf.cpu(), M, I).unsqueeze(-1))
    assert rel_err(o_deq.view(M, I), want_mx) < 6e-2
