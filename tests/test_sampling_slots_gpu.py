"""The cluster sampler (csrc/kernels/sampling_cluster.cu) against the fp32 PyTorch oracle:
bf16 and fp32 logits, and slot mode, where penalties, logit bias and min_tokens come from
device tables that the kernel itself advances after each draw."""
import numpy as np
import pytest
import torch

from rusteeze_b200 import ops
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.engine.sampler import SampleRow, Sampler
from rusteeze_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _Seq:
    """The fields of an engine Sequence that sampling reads."""
    _ids = iter(range(10 ** 6, 10 ** 7))

    def __init__(self, prompt, out=()):
        self.seq_id = next(self._ids)
        self.token_ids = list(prompt) + list(out)
        self.prompt_len = len(prompt)

    @property
    def output_token_ids(self):
        return self.token_ids[self.prompt_len:]


def _tie_inclusive_probs(logits, T, k, p, mp):
    """Filtered, renormalised probabilities where tokens that tie with the boundary are all
    kept (the kernel selects on the value, so equal values share a fate; bf16 logits tie
    often): keep t when fewer than k tokens are strictly more likely, the mass of strictly
    more likely tokens is < p, and p_t >= mp * p_max."""
    x = logits.float() / T
    probs = torch.softmax(x, -1)
    out = torch.zeros_like(probs)
    for r in range(probs.shape[0]):
        pr = probs[r]
        sp, _ = pr.sort(descending=True)
        uniq, inv, counts = torch.unique_consecutive(sp, return_inverse=True, return_counts=True)
        n_above = torch.cumsum(counts, 0) - counts                    # tokens strictly above each value
        m_above = torch.cumsum(uniq * counts, 0) - uniq * counts      # their mass
        keep_v = (n_above < (k if k > 0 else pr.numel())) & (m_above < p) & (uniq >= mp * sp[0])
        thr = uniq[keep_v].min()
        keep = pr >= thr
        out[r] = torch.where(keep, pr, torch.zeros_like(pr))
        out[r] /= out[r].sum()
    return out


def _rows(n, V, **kw):
    rng = np.random.default_rng(0)
    rows = []
    for i in range(n):
        s = _Seq(rng.integers(0, V, 40).tolist(), rng.integers(0, V, 7).tolist())
        p = SamplingParams(**kw)
        rows.append(SampleRow(p, None, None, 1000 + i, len(s.output_token_ids), (2,), None, s, 0))
    return rows


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("V", [128256, 32000, 1000, 16])
def test_greedy_rows_exact(dtype, V):
    torch.manual_seed(3)
    logits = (torch.randn(70, V, device=DEV) * 2).to(dtype)
    tok, lp = ops.sample(logits, None, None, None, None, None, None, greedy_all=True)
    x = logits.float()
    assert torch.equal(tok, x.argmax(-1))
    ref_lp = torch.log_softmax(x, -1).gather(1, tok.view(-1, 1)).view(-1)
    assert torch.allclose(lp, ref_lp, atol=2e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_bf16_and_fp32_rows_sample_the_same_support(dtype):
    torch.manual_seed(4)
    B, V = 128, 128256
    logits = (torch.randn(B, V, device=DEV) * 3).to(dtype)
    f = lambda v, dt: torch.full((B,), v, dtype=dt, device=DEV)  # noqa: E731
    tok, lp = ops.sample(logits, f(0.8, torch.float32), f(40, torch.int32), f(0.9, torch.float32),
                         f(0.0, torch.float32), torch.arange(B, device=DEV, dtype=torch.int64), f(5, torch.int64),
                         greedy_all=False)
    probs = _tie_inclusive_probs(logits.float().cpu(), 0.8, 40, 0.9, 0.0)
    chosen = probs.gather(1, tok.cpu().view(-1, 1)).view(-1)
    assert (chosen > 0).all()
    full = torch.log_softmax(logits.float().cpu() / 0.8, -1).gather(1, tok.cpu().view(-1, 1)).view(-1)
    assert torch.allclose(lp.cpu(), full, atol=2e-3)


def test_slot_mode_penalties_bias_and_min_tokens_match_the_oracle():
    """Greedy rows with repetition / frequency / presence penalties, logit bias and
    min_tokens: the kernel's choice equals the argmax of the oracle's processed logits;
    then the kernel's own count update makes a huge frequency penalty forbid the token
    it just chose, and min_tokens stops masking EOS once enough tokens were drawn."""
    torch.manual_seed(5)
    V = 32000
    S = Sampler(V)
    S.max_slots = 64
    rows = _rows(6, V, temperature=0.0, repetition_penalty=1.3, frequency_penalty=0.5, presence_penalty=0.4,
                 logit_bias={7: 5.0, 11: -3.0}, max_tokens=20)
    logits = torch.randn(6, V, device=DEV) * 2
    h = S.launch(logits, rows)
    res = S.finish(h)
    x = logits.cpu()
    pen = ref.apply_penalties(x, [list(r.output_ids) for r in rows], [list(r.prompt_ids) for r in rows],
                              torch.full((6,), 1.3), torch.full((6,), 0.5), torch.full((6,), 0.4))
    pen[:, 7] += 5.0
    pen[:, 11] -= 3.0
    assert res.tokens == pen.argmax(-1).tolist()
    # second step, same slots: frequency penalty 2.0 per count on the chosen token
    rows2 = _rows(1, V, temperature=0.0, frequency_penalty=2.0, max_tokens=20)
    one = torch.zeros(1, V, device=DEV)
    one[0, 123] = 1.5
    t1 = S.finish(S.launch(one, rows2)).tokens[0]
    t2 = S.finish(S.launch(one, rows2)).tokens[0]
    assert t1 == 123 and t2 != 123           # the kernel counted its own draw
    # min_tokens: EOS (id 2) masked for the first 2 draws of this slot, then allowed
    rows3 = _rows(1, V, temperature=0.0, min_tokens=2, max_tokens=20)
    rows3[0].offset = 0
    eos = torch.zeros(1, V, device=DEV)
    eos[0, 2] = 10.0
    got = [S.finish(S.launch(eos, rows3)).tokens[0] for _ in range(3)]
    assert got[0] != 2 and got[1] != 2 and got[2] == 2


def test_slot_mode_sampled_rows_stay_in_the_filtered_support_and_advance_the_stream():
    torch.manual_seed(6)
    V = 128256
    S = Sampler(V)
    S.max_slots = 300
    rows = _rows(256, V, temperature=0.7, top_p=0.9, max_tokens=20)
    logits = (torch.randn(256, V, device=DEV) * 3).to(torch.bfloat16)
    a = S.finish(S.launch(logits, rows))
    probs = _tie_inclusive_probs(logits.float().cpu(), 0.7, -1, 0.9, 0.0)
    chosen = probs.gather(1, torch.tensor(a.tokens).view(-1, 1)).view(-1)
    assert (chosen > 0).all()
    full = torch.log_softmax(logits.float().cpu() / 0.7, -1).gather(1, torch.tensor(a.tokens).view(-1, 1)).view(-1)
    assert np.allclose(np.array(a.logprobs), full.numpy(), atol=2e-3)
    b = S.finish(S.launch(logits, rows))     # the slots' generated counts advanced: new draws
    assert a.tokens != b.tokens
    for r in rows:
        S.release(r.seq.seq_id)
    assert len(S._slots.free) == 300


def test_growing_vocabulary_in_one_process():
    """The kernel's shared memory grows with the vocabulary: a small-vocabulary launch
    followed by a large one in the same process must raise the kernel's opt-in."""
    torch.manual_seed(7)
    for V in (1000, 32000, 128256, 152064):
        logits = torch.randn(4, V, device=DEV)
        tok, _ = ops.sample(logits, None, None, None, None, None, None, greedy_all=True)
        assert torch.equal(tok, logits.argmax(-1))


def test_top_k_and_top_p_draws_follow_the_filtered_distribution():
    """Chi-square of many draws of one row against the filtered, renormalised oracle:
    top-k (several rejection rounds on a flat row) and top-p."""
    V = 64
    torch.manual_seed(9)
    base = torch.randn(V) * 0.5
    for T, k, p in ((1.0, 5, 1.0), (0.8, -1, 0.6), (1.2, 12, 0.7)):
        N = 8192
        logits = base.to(DEV).repeat(N, 1)
        f = lambda v, dt: torch.full((N,), v, dtype=dt, device=DEV)  # noqa: E731
        tok, _ = ops.sample(logits, f(T, torch.float32), f(k, torch.int32), f(p, torch.float32),
                            f(0.0, torch.float32), torch.arange(N, device=DEV, dtype=torch.int64), f(3, torch.int64),
                            greedy_all=False)
        probs = _tie_inclusive_probs(base.unsqueeze(0), T, k, p, 0.0)[0]
        cnt = torch.bincount(tok.cpu(), minlength=V).float()
        exp = probs * N
        keep = exp > 0
        assert (cnt[~keep] == 0).all(), (T, k, p)
        chi2 = (((cnt - exp) ** 2)[keep] / exp[keep]).sum().item()
        assert chi2 < 3 * int(keep.sum()) + 20, (T, k, p, chi2)
