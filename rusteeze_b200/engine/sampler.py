"""Batched token sampling.

Semantics follow the reference sampler (crates/rusteeze-engine/src/
sampler.rs:56-244): repetition penalty over previously seen tokens, logit
bias, then greedy (temperature 0 or top_k 1), or temperature -> softmax ->
top-k -> top-p over the (not renormalised) top-k probabilities -> renormalise
-> draw; Mirostat v1/v2 (sampler.rs:181-244).  Added here: frequency and
presence penalties (simd_ops.rs:104-119 defines them, the reference never
applies them), min-p, min_tokens (EOS masked until reached), per-request
seeds (the reference reseeds every row with `i ^ 0xDEADBEEF` each call,
parallel_sampler.rs:86-89), and logprobs.

On the GPU the whole batch is sampled by one kernel launch (sm_100a
`topk_topp_sample`: per-row max/normaliser, histogram threshold selection
for top-k/top-p/min-p, Gumbel-max draw from a counter-based Philox stream
keyed by (seed, step)), or `argmax_sample` when every row is greedy.  Guided
rows have their excluded tokens set to -inf first and are sampled with the rest.
Rows that need Mirostat, typical-p or eta/epsilon cutoffs are copied to the host
and sampled there.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence as Seq, Tuple

import numpy as np
import torch

from rusteeze_b200 import ops
from rusteeze_b200.utils.op_timer import OP_TIMER
from rusteeze_b200.core.sampling_params import SamplingParams
from rusteeze_b200.ops import reference as ref

_MASK = -1e30


class SampleRow:
    """One row of logits to sample.  `seq` (the engine's Sequence, when there is one) and
    `sub` (the sample index of a best_of prompt row) key the row's device slot; the token
    histories that penalties read are taken from the sequence only when they are needed."""
    __slots__ = ("params", "_prompt_ids", "_output_ids", "seed", "offset", "eos_ids", "mirostat_mu", "seq", "sub",
                 "allowed")

    def __init__(self, params: SamplingParams, prompt_ids: Optional[Seq[int]] = None,
                 output_ids: Optional[Seq[int]] = None, seed: int = 0, offset: int = 0,
                 eos_ids: Tuple[int, ...] = (), mirostat_mu: Optional[float] = None, seq=None, sub: int = 0):
        self.params = params
        self._prompt_ids = prompt_ids
        self._output_ids = output_ids
        self.seed, self.offset, self.eos_ids, self.mirostat_mu = seed, offset, eos_ids, mirostat_mu
        self.seq, self.sub = seq, sub
        self.allowed = None            # guided decoding: bool mask [vocab] of the tokens that may come next

    @property
    def prompt_ids(self) -> Seq[int]:
        if self._prompt_ids is None:
            self._prompt_ids = self.seq.token_ids[:self.seq.prompt_len] if self.seq is not None else ()
        return self._prompt_ids

    @property
    def output_ids(self) -> Seq[int]:
        if self._output_ids is None:
            self._output_ids = self.seq.output_token_ids if self.seq is not None else ()
        return self._output_ids


class SlotTable:
    """Device-resident sampling state, one slot per live sequence (see
    csrc/kernels/sampling_cluster.cu): parameters uploaded once when a sequence is first
    sampled (or again after a preemption), the generated-token counter the kernel
    advances, and for sequences with penalties a prompt bitmask and 16-bit output
    counts the kernel updates after each draw.  A step then only uploads one int32 per
    row (slot | sample index << 16).

    Slots are released when a sequence finishes or is preempted; the next owner's
    parameters are written by a kernel launched after every step that could still
    touch the old owner, so stream order protects the hand-over."""

    def __init__(self, max_slots: int, vocab: int, device: torch.device):
        C = ops.cuda_ext()
        self.MAXB, self.MAXS = int(C.SAMPLE_MAX_BIAS), int(C.SAMPLE_MAX_STOP)
        S, self.V, self.dev = max_slots, vocab, device
        z = lambda *sh, dt=torch.int32: torch.zeros(*sh, dtype=dt, device=device)  # noqa: E731
        self.f32 = z(S, 8, dt=torch.float32)
        self.i32 = z(S, 8)
        self.n_gen = z(S)
        self.seed = z(S, dt=torch.int64)
        self.cnt = z(0)
        self.seen = z(0)
        self.bias_tok = z(S, self.MAXB)
        self.bias_val = z(S, self.MAXB, dt=torch.float32)
        self.stop_ids = z(S, self.MAXS)
        self.free = list(range(S - 1, -1, -1))
        self.of: Dict[int, int] = {}            # seq id -> slot
        self.pen_of: Dict[int, int] = {}        # slot -> penalty row
        self.pen_free: List[int] = []
        self._pin_info = [torch.empty(1 << 14, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._pk = 0
        self.uploads = 0

    def tables(self) -> List[torch.Tensor]:
        return [self.f32, self.i32, self.n_gen, self.seed, self.cnt, self.seen, self.bias_tok, self.bias_val,
                self.stop_ids]

    def fits(self, row: SampleRow) -> bool:
        p = row.params
        return (len(p.logit_bias) <= self.MAXB and len(row.eos_ids) + len(p.stop_token_ids) <= self.MAXS)

    def release(self, seq_id: int) -> None:
        slot = self.of.pop(seq_id, None)
        if slot is None:
            return
        pr = self.pen_of.pop(slot, None)
        if pr is not None:
            self.pen_free.append(pr)
        self.free.append(slot)

    def _pen_row(self, slot: int) -> int:
        if self.cnt.numel() == 0:
            P = self.f32.shape[0]
            self.cnt = torch.zeros(P, (self.V + 1) // 2, dtype=torch.int32, device=self.dev)
            self.seen = torch.zeros(P, (self.V + 31) // 32, dtype=torch.int32, device=self.dev)
            self.pen_free = list(range(P - 1, -1, -1))
        pr = self.pen_free.pop()
        self.pen_of[slot] = pr
        return pr

    def row_info(self, rows: List[SampleRow]) -> torch.Tensor:
        """Slot of every row (assigning and uploading new ones); returns the device int32
        row-info vector for `ops.sample_slots`."""
        R = len(rows)
        info = np.empty(R, dtype=np.int32)
        new: List[Tuple[int, SampleRow]] = []
        for i, r in enumerate(rows):
            key = r.seq.seq_id
            slot = self.of.get(key)
            if slot is None:
                if not self.free:
                    raise RuntimeError("no free sampling slot (more live sequences than slots)")
                slot = self.free.pop()
                self.of[key] = slot
                new.append((slot, r))
            info[i] = slot | (r.sub << 16)
        if new:
            self._upload(new)
        buf = self._pin_info[self._pk]
        self._pk ^= 1
        if R > buf.numel():
            raise ValueError("too many sample rows for the row-info buffer")
        buf[:R].copy_(torch.from_numpy(info))
        return buf[:R].to(self.dev, non_blocking=True)

    def _upload(self, new: List[Tuple[int, SampleRow]]) -> None:
        n = len(new)
        B, S = self.MAXB, self.MAXS
        slot = np.empty(n, dtype=np.int32)
        f32 = np.zeros((n, 8), dtype=np.float32)
        i32 = np.zeros((n, 8), dtype=np.int32)
        n_gen = np.empty(n, dtype=np.int32)
        seed = np.empty(n, dtype=np.int64)
        btok = np.zeros((n, B), dtype=np.int32)
        bval = np.zeros((n, B), dtype=np.float32)
        stops = np.zeros((n, S), dtype=np.int32)
        off = [0]
        toks: List[int] = []
        for i, (sl, r) in enumerate(new):
            p = r.params
            slot[i] = sl
            f32[i, :6] = (0.0 if p.is_greedy else p.temperature, p.top_p, p.min_p, p.repetition_penalty,
                          p.frequency_penalty, p.presence_penalty)
            pen = self._pen_row(sl) if p.has_penalties() else -1
            st = list(r.eos_ids) + list(p.stop_token_ids)
            i32[i, :5] = (p.top_k, p.min_tokens, pen, len(p.logit_bias), len(st))
            n_gen[i] = r.offset
            seed[i] = (r.seed - 7919 * r.sub) & ((1 << 63) - 1)    # the row adds 7919 * sub back
            if p.logit_bias:
                btok[i, :len(p.logit_bias)] = list(p.logit_bias.keys())
                bval[i, :len(p.logit_bias)] = list(p.logit_bias.values())
            if st:
                stops[i, :len(st)] = st
            if pen >= 0:
                toks += list(r.prompt_ids)
                off.append(len(toks))
                toks += list(r.output_ids)
                off.append(len(toks))
            else:
                off += [len(toks), len(toks)]
        d = lambda a: torch.from_numpy(a).pin_memory().to(self.dev, non_blocking=True)  # noqa: E731
        tk = d(np.asarray(toks if toks else [0], dtype=np.int32))
        ops.cuda_ext().sample_slot_init(self.tables(), n, self.V, d(slot), d(f32), d(i32), d(n_gen), d(seed),
                                        d(btok), d(bval), d(stops), d(np.asarray(off, dtype=np.int32)), tk)
        ops.add_launches(1)
        self.uploads += n


@dataclass
class AsyncSample:
    tokens: torch.Tensor          # device int64 [R]: next step's pending input ids
    host: object                  # pinned (int64 token ids, fp32 logprobs), each >= R long
    rows: int
    event: "torch.cuda.Event"
    result: Optional["SampleResult"] = None    # host-sampled rows (CPU engines): already known


@dataclass
class SampleResult:
    tokens: List[int]
    logprobs: List[Optional[float]]
    top_logprobs: List[Optional[Dict[int, float]]]
    mirostat_mu: List[Optional[float]]


def _philox_like_seed(seed: int, offset: int) -> int:
    x = (seed * 0x9E3779B97F4A7C15 + offset * 0xBF58476D1CE4E5B9) & ((1 << 63) - 1)
    return x


class Sampler:
    def __init__(self, vocab_size: int):
        self.vocab_size = vocab_size
        self._param_cache: Dict[Tuple, Tuple[torch.Tensor, ...]] = {}
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0

    # ------------------------------------------------------------------ pre-processing
    def _process_logits(self, logits: torch.Tensor, rows: List[SampleRow]) -> torch.Tensor:
        """Penalties, logit bias, min_tokens masking (in place when possible)."""
        need_pen = [i for i, r in enumerate(rows) if r.params.has_penalties()]
        if need_pen:
            sub = logits[need_pen]
            sub_cpu_rows = [rows[i] for i in need_pen]
            rep = torch.tensor([r.params.repetition_penalty for r in sub_cpu_rows])
            freq = torch.tensor([r.params.frequency_penalty for r in sub_cpu_rows])
            pres = torch.tensor([r.params.presence_penalty for r in sub_cpu_rows])
            if logits.is_cuda:
                sub = _apply_penalties_device(sub, sub_cpu_rows, rep, freq, pres)
            else:
                sub = ref.apply_penalties(sub, [list(r.output_ids) for r in sub_cpu_rows],
                                          [list(r.prompt_ids) for r in sub_cpu_rows], rep, freq, pres)
            logits[need_pen] = sub
        for i, r in enumerate(rows):
            p = r.params
            if p.logit_bias:
                idx = torch.tensor(list(p.logit_bias.keys()), dtype=torch.long, device=logits.device)
                val = torch.tensor(list(p.logit_bias.values()), dtype=logits.dtype, device=logits.device)
                logits[i].index_add_(0, idx, val)
            if p.min_tokens and r.offset < p.min_tokens:     # offset == tokens generated so far
                stop = list(r.eos_ids) + list(p.stop_token_ids)
                if stop:
                    logits[i, torch.tensor(stop, device=logits.device)] = _MASK
        return logits

    # ------------------------------------------------------------------ asynchronous entry
    @staticmethod
    def async_eligible(params: SamplingParams) -> bool:
        """Rows whose sampling runs entirely in the GPU kernel with nothing to read back
        but (token, logprob): penalties, logit bias (up to the slot table's 320 entries)
        and min_tokens (up to 32 stop ids with EOS) live in the device slot tables; host
        samplers and top logprobs do not."""
        return (not params.needs_host_sampling() and params.logprobs is None and params.prompt_logprobs is None
                and params.guided_decoding is None
                and len(params.logit_bias) <= 320 and len(params.stop_token_ids) <= 48)

    def slots(self, device, max_slots: int) -> SlotTable:
        if getattr(self, "_slots", None) is None:
            self._slots = SlotTable(max_slots, self.vocab_size, device)
        return self._slots

    def release(self, seq_id: int) -> None:
        """A sequence finished, was aborted or preempted: its device slot is free."""
        st = getattr(self, "_slots", None)
        if st is not None:
            st.release(seq_id)

    def _drop_slots(self) -> None:
        """A synchronous step samples with host-built parameters and advances no slot
        counters: every slot is released, so the next pipelined step re-uploads fresh
        state (generated counts, penalty histories) for the sequences it samples."""
        st = getattr(self, "_slots", None)
        if st is not None and st.of:
            for k in list(st.of):
                st.release(k)

    def launch(self, logits: torch.Tensor, rows: List[SampleRow]) -> "AsyncSample":
        """Enqueues the sampling kernel and the copy of its results into pinned
        host memory; `finish` waits for them.  Device rows only."""
        R = logits.shape[0]
        self.last_h2d_bytes = 0
        if not logits.is_cuda:
            # CPU engines (tests of the pipelined schedule): sample now, hand back the same handle
            res = self.sample(logits, rows)
            return AsyncSample(torch.tensor(res.tokens, dtype=torch.int64), None, R, None, res)
        with OP_TIMER.section("sample"):
            st = self.slots(logits.device, self.max_slots) if getattr(self, "max_slots", 0) else None
            if st is not None and all(r.seq is not None and st.fits(r) for r in rows):
                info = st.row_info(rows)
                self.last_h2d_bytes += 4 * R
                toks, lp = ops.sample_slots(logits, info, st.tables())
            else:
                toks, lp = self._sample_device_async(logits, rows)
        # every host staging buffer is 1-D and only used through contiguous
        # prefixes: a strided pinned slice would make torch stage the copy
        # through a blocking temporary
        if not hasattr(self, "_pinned"):
            # (token ids, logprobs) per set: two plain device-to-host copies, no packing kernel
            self._pinned = [(torch.empty(1 << 15, dtype=torch.int64, pin_memory=True),
                             torch.empty(1 << 15, dtype=torch.float32, pin_memory=True)) for _ in range(2)]
            self._pk = 0
        bt, bl = self._pinned[self._pk]
        self._pk ^= 1
        if R > bt.numel():
            raise ValueError("too many sample rows for the async readback buffer")
        bt[:R].copy_(toks, non_blocking=True)
        bl[:R].copy_(lp, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        return AsyncSample(toks, (bt, bl), R, ev)

    def finish(self, a: "AsyncSample") -> SampleResult:
        if a.result is not None:
            self.last_d2h_bytes = 0
            return a.result
        a.event.synchronize()
        R = a.rows
        self.last_d2h_bytes = 12 * R
        bt, bl = a.host
        return SampleResult(bt[:R].tolist(), bl[:R].tolist(), [None] * R, [None] * R)

    def _sample_device_async(self, logits: torch.Tensor, rows: List[SampleRow]):
        greedy = [r.params.is_greedy for r in rows]
        if all(greedy):
            return ops.sample(logits, None, None, None, None, None, None, greedy_all=True, want_logprobs=False)
        dev = logits.device
        R = len(rows)
        if not hasattr(self, "_param_pin"):
            self._param_pin = [(torch.empty(4 << 14, dtype=torch.float32, pin_memory=True),
                                torch.empty(2 << 14, dtype=torch.int64, pin_memory=True)) for _ in range(2)]
            self._ppk = 0
        hf, hi = self._param_pin[self._ppk]
        self._ppk ^= 1
        if R > (1 << 14):
            raise ValueError("too many sample rows for the async parameter buffer")
        f = np.empty(4 * R, dtype=np.float32)
        f[:R] = [0.0 if g else r.params.temperature for g, r in zip(greedy, rows)]
        f[R:2 * R] = [r.params.top_k for r in rows]
        f[2 * R:3 * R] = [r.params.top_p for r in rows]
        f[3 * R:] = [r.params.min_p for r in rows]
        hf[:4 * R].copy_(torch.from_numpy(f))
        hi[:2 * R].copy_(torch.from_numpy(np.asarray([r.seed & ((1 << 63) - 1) for r in rows] +
                                                     [r.offset for r in rows], dtype=np.int64)))
        d = hf[:4 * R].to(dev, non_blocking=True)
        di = hi[:2 * R].to(dev, non_blocking=True)
        self.last_h2d_bytes += 32 * R
        return ops.sample(logits, d[:R], d[R:2 * R].int(), d[2 * R:3 * R], d[3 * R:], di[:R], di[R:],
                          greedy_all=False, want_logprobs=False)

    # ------------------------------------------------------------------ main entry
    def sample(self, logits: torch.Tensor, rows: List[SampleRow]) -> SampleResult:
        """logits: fp32 [R, V] (device or host), one row per SampleRow."""
        R = logits.shape[0]
        assert R == len(rows)
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0
        self._drop_slots()
        # the host-side rules index the logits in place: fp32 (the GPU path hands bf16 views)
        logits = logits.float()
        logits = self._process_logits(logits, rows)
        _apply_guides(logits, rows)
        host_rows = [i for i, r in enumerate(rows) if r.params.needs_host_sampling()]
        tokens: List[int] = [0] * R
        lps: List[Optional[float]] = [None] * R
        mus: List[Optional[float]] = [None] * R
        dev_rows = [i for i in range(R) if i not in set(host_rows)] if host_rows else list(range(R))
        if dev_rows:
            sub = logits if len(dev_rows) == R else logits[dev_rows]
            with OP_TIMER.section("sample"):
                t, lp = self._sample_device(sub, [rows[i] for i in dev_rows])
            for j, i in enumerate(dev_rows):
                tokens[i] = t[j]
                lps[i] = lp[j]
        for i in host_rows:
            tok, lp, mu = _host_sample(logits[i].float().cpu(), rows[i])
            tokens[i], lps[i], mus[i] = tok, lp, mu
        tops: List[Optional[Dict[int, float]]] = [None] * R
        want = [i for i, r in enumerate(rows) if r.params.logprobs is not None]
        if want:
            lsm = torch.log_softmax(logits[want].float(), dim=-1)
            for j, i in enumerate(want):
                k = rows[i].params.logprobs
                d: Dict[int, float] = {}
                if k:
                    v, ix = lsm[j].topk(min(k, lsm.shape[1]))
                    d = dict(zip(ix.tolist(), v.tolist()))
                d[tokens[i]] = float(lsm[j, tokens[i]])
                tops[i] = d
                lps[i] = d[tokens[i]]
        return SampleResult(tokens, lps, tops, mus)

    def _sample_device(self, logits: torch.Tensor, rows: List[SampleRow]):
        R = logits.shape[0]
        greedy = [r.params.is_greedy for r in rows]
        if not logits.is_cuda:
            return _cpu_sample(logits, rows)
        dev = logits.device
        want_lp = any(r.params.logprobs is not None for r in rows)
        if all(greedy):
            toks, lp = ops.sample(logits, None, None, None, None, None, None, greedy_all=True,
                                  want_logprobs=want_lp)
        else:
            temp = torch.tensor([0.0 if g else r.params.temperature for g, r in zip(greedy, rows)],
                                dtype=torch.float32)
            top_k = torch.tensor([r.params.top_k for r in rows], dtype=torch.int32)
            top_p = torch.tensor([r.params.top_p for r in rows], dtype=torch.float32)
            min_p = torch.tensor([r.params.min_p for r in rows], dtype=torch.float32)
            seeds = torch.tensor([r.seed & ((1 << 63) - 1) for r in rows], dtype=torch.int64)
            offs = torch.tensor([r.offset for r in rows], dtype=torch.int64)
            packed = [x.pin_memory().to(dev, non_blocking=True) for x in (temp, top_k, top_p, min_p, seeds, offs)]
            self.last_h2d_bytes += sum(x.numel() * x.element_size() for x in packed)
            toks, lp = ops.sample(logits, *packed, greedy_all=False, want_logprobs=want_lp)
        both = torch.stack([toks.double(), lp.double()]).cpu()
        self.last_d2h_bytes += both.numel() * 8
        return [int(x) for x in both[0].tolist()], both[1].tolist()


def _apply_guides(logits: torch.Tensor, rows: List[SampleRow]) -> None:
    """Guided decoding: tokens outside each guided row's `allowed` mask get -inf, in place,
    so the batched sampler (the GPU kernel, or its host restatement) draws only allowed
    tokens with the row's own temperature / top-k / top-p / min-p."""
    idx = [i for i, r in enumerate(rows) if r.allowed is not None and r.allowed.any()]
    if not idx:
        return
    V = logits.shape[1]
    m = torch.from_numpy(np.stack([rows[i].allowed[:V] for i in idx]))
    dev = logits.device
    sel = torch.tensor(idx, dtype=torch.long, device=dev)
    sub = logits.index_select(0, sel)
    sub.masked_fill_(~m.to(dev), float("-inf"))
    logits.index_copy_(0, sel, sub)


def _apply_penalties_device(sub: torch.Tensor, rows: List[SampleRow], rep, freq, pres) -> torch.Tensor:
    dev = sub.device
    V = sub.shape[1]
    for j, r in enumerate(rows):
        p = r.params
        row = sub[j]
        if p.repetition_penalty != 1.0:
            seen = torch.tensor(sorted(set(r.prompt_ids) | set(r.output_ids)), dtype=torch.long, device=dev)
            if seen.numel():
                v = row[seen]
                row[seen] = torch.where(v > 0, v / p.repetition_penalty, v * p.repetition_penalty)
        if r.output_ids and (p.frequency_penalty or p.presence_penalty):
            cnt = torch.bincount(torch.tensor(list(r.output_ids), dtype=torch.long, device=dev),
                                 minlength=V).float()
            row -= p.frequency_penalty * cnt + p.presence_penalty * (cnt > 0).float()
    return sub


def _row_generator(seed: int, offset: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(_philox_like_seed(seed, offset))
    return g


def _cpu_sample(logits: torch.Tensor, rows: List[SampleRow]):
    toks, lps = [], []
    for i, r in enumerate(rows):
        x = logits[i].float()
        if r.params.is_greedy:
            t = int(torch.argmax(x))
            toks.append(t)
            lps.append(float(torch.log_softmax(x, -1)[t]))
            continue
        p = r.params
        probs = ref.topk_topp_minp_probs(x.unsqueeze(0), torch.tensor([p.temperature]),
                                         torch.tensor([p.top_k]), torch.tensor([p.top_p]),
                                         torch.tensor([p.min_p]))[0]
        t = int(torch.multinomial(probs, 1, generator=_row_generator(r.seed, r.offset)))
        toks.append(t)
        lps.append(math.log(max(float(probs[t]), 1e-45)))
    return toks, lps


def _host_sample(x: torch.Tensor, r: SampleRow):
    """Rows the GPU kernel does not cover: guided decoding (the row's `allowed` mask,
    applied to the logits first, like a logits processor), Mirostat v1/v2, typical-p,
    eta / epsilon cutoffs; then top-k / top-p / min-p of the remaining distribution."""
    p = r.params
    g = _row_generator(r.seed, r.offset)
    if r.allowed is not None:
        allowed = torch.from_numpy(r.allowed[:x.shape[0]])
        if bool(allowed.any()):
            x = x.masked_fill(~allowed, float("-inf"))
    if p.temperature > 0:
        x = x / p.temperature
    probs = torch.softmax(x, -1)
    if p.mirostat_mode:
        mu = r.mirostat_mu if r.mirostat_mu is not None else 2.0 * p.mirostat_tau
        sp, si = probs.sort(descending=True)
        if p.mirostat_mode == 1:
            k = max(1, min(int(math.exp(min(mu, 50.0))), sp.numel()))
            cand, idx = sp[:k], si[:k]
        else:
            keep = -torch.log(sp.clamp_min(1e-30)) <= mu
            if not keep.any():
                keep[0] = True
            cand, idx = sp[keep], si[keep]
        cand = cand / cand.sum()
        j = int(torch.multinomial(cand, 1, generator=g))
        tok, pr = int(idx[j]), float(cand[j])
        surprise = -math.log(max(pr, 1e-10))
        mu = mu + p.mirostat_eta * (p.mirostat_tau - surprise)
        return tok, math.log(max(pr, 1e-45)), mu
    keep = torch.isfinite(x)
    if p.typical_p > 0:
        ent = -(probs * torch.log(probs.clamp_min(1e-30))).sum()
        dev = (-torch.log(probs.clamp_min(1e-30)) - ent).abs()
        order = dev.argsort()
        cum = probs[order].cumsum(0)
        n = int((cum < p.typical_p).sum()) + 1
        m = torch.zeros_like(keep)
        m[order[:n]] = True
        keep &= m
    if p.epsilon_cutoff > 0:
        keep &= probs >= p.epsilon_cutoff
    if p.eta_cutoff > 0:
        ent = -(probs * torch.log(probs.clamp_min(1e-30))).sum()
        eps = min(p.eta_cutoff, math.sqrt(p.eta_cutoff) * math.exp(-float(ent)))
        keep &= probs >= eps
    if p.temperature > 0 and (p.top_k > 0 or p.top_p < 1.0 or p.min_p > 0.0):
        fp = ref.topk_topp_minp_probs(x.unsqueeze(0), torch.ones(1), torch.tensor([p.top_k]),
                                      torch.tensor([p.top_p]), torch.tensor([p.min_p]))[0]
        keep &= fp > 0
    if not keep.any():
        keep[int(x.argmax())] = True
    pr = torch.where(keep, probs, torch.zeros_like(probs))
    if float(pr.sum()) <= 0.0:
        # every kept token's probability underflowed (or was masked, e.g. EOS before
        # min_tokens when the constraint allows nothing else): the best kept logit
        tok = int(torch.where(keep, x, torch.full_like(x, -float("inf"))).argmax())
        return tok, math.log(max(float(probs[tok]), 1e-45)), None
    if p.temperature == 0:
        tok = int(pr.argmax())
    else:
        pr = pr / pr.sum()
        tok = int(torch.multinomial(pr, 1, generator=g))
    return tok, math.log(max(float(probs[tok]), 1e-45)), None
