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
    probs = ref.topk_topp_minp_probs(logits.float().cpu(), torch.full((B,), 0.8), torch.full((B,), 40),
                                     torch.full((B,), 0.9), torch.full((B,), 0.0))
    chosen = probs.gather(1, tok.cpu().view(-1, 1)).view(-1)
    assert (chosen > 0).all()
    assert ((lp.cpu() - chosen.log()).abs() < 2e-2).all()


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
    probs = ref.topk_topp_minp_probs(logits.float().cpu(), torch.full((256,), 0.7), torch.full((256,), -1),
                                     torch.full((256,), 0.9), torch.full((256,), 0.0))
    chosen = probs.gather(1, torch.tensor(a.tokens).view(-1, 1)).view(-1)
    assert (chosen > 0).all()
    assert (np.abs(np.array(a.logprobs) - chosen.log().numpy()) < 2e-2).all()
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
