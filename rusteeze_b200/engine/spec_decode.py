"""Draft-model speculative decoding.

The reference ships an unused tree-speculation module whose acceptance rule
(`target logit > top * threshold`, crates/rusteeze-engine/src/speculative.rs:
291-348) does not preserve the target distribution.  Here:

  * a draft model (e.g. a 1B Llama-3.2-like model next to Llama-3-70B)
    keeps its own KV cache, indexed by the SAME block ids as the target
    (the scheduler reserves k lookahead slots per decoding sequence);
  * each pure-decode step runs k batched draft steps, then ONE target
    forward over k+1 positions per sequence (the varlen paged attention
    kernel with q_len = k+1), then the sm_100a `spec_verify` kernel:
    greedy requests accept the longest prefix matching the target argmax;
    sampled requests use standard rejection sampling (accept d with
    probability min(1, p(d)/q(d)), resample from normalise(max(0, p-q)),
    bonus token from p after k accepts) -- the emitted tokens follow the
    target distribution exactly;
  * rollback is implicit: a sequence's computed length advances by
    accepted+1, so KV written for rejected positions is simply overwritten
    later; the draft re-feeds the tokens it has not cached (1, or 2 after a
    full accept) at the start of the next round;
  * steps that contain prefill chunks run normally on the target and the
    draft processes the same tokens to stay in sync.
Sampled speculation applies temperature only (top-k/top-p requests fall
back to plain decoding).

`method: ngram` replaces the draft model by prompt lookup (the n-gram method the
reference's configuration names, crates/rusteeze-core/src/config.rs:635-645, without
an implementation): each sequence proposes the k tokens that followed the most recent
earlier occurrence of its last n tokens (C++ `_host.ngram_propose`, longest n first).
There is no draft KV and no draft forward; the target pass and the greedy verify are
the same as above, so the emitted tokens equal plain greedy decoding.  A proposal is a
point mass, not a distribution, so n-gram rounds run for greedy batches only (sampled
requests decode normally), and a step in which no sequence has a proposal runs as a
plain step.
"""
from __future__ import annotations

import dataclasses
import logging
import time
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from rusteeze_b200 import ops
from rusteeze_b200.engine.model_runner import ModelRunner
from rusteeze_b200.models.config import ModelConfig, get_preset
from rusteeze_b200.models.loader import build_model

log = logging.getLogger("rusteeze.spec")


def _verify_cpu(target: torch.Tensor, draft_logits, draft: torch.Tensor, temps, seeds, offsets):
    """Host restatement of the verify kernel (greedy exact; sampled via torch RNG)."""
    B, k = draft.shape
    V = target.shape[1]
    out = torch.full((B, k + 1), -1, dtype=torch.long)
    acc = torch.zeros(B, dtype=torch.long)
    for b in range(B):
        g = torch.Generator().manual_seed((int(seeds[b]) * 1000003 + int(offsets[b])) & ((1 << 63) - 1))
        for j in range(k + 1):
            t = target[b * (k + 1) + j].float()
            if temps[b] <= 0:
                a = int(t.argmax())
                if j < k and a == int(draft[b, j]):
                    out[b, j] = a
                    acc[b] += 1
                    continue
                out[b, j] = a
                break
            p = torch.softmax(t / temps[b], -1)
            if j < k:
                q = torch.softmax(draft_logits[b * k + j].float() / temps[b], -1)
                d = int(draft[b, j])
                if torch.rand((), generator=g) * q[d] < p[d]:
                    out[b, j] = d
                    acc[b] += 1
                    continue
                r = (p - q).clamp_min(0)
                out[b, j] = int(torch.multinomial(r / r.sum(), 1, generator=g)) if r.sum() > 0 else d
                break
            out[b, j] = int(torch.multinomial(p, 1, generator=g))
    return acc, out


def draft_model_config(target: ModelConfig, spec_cfg) -> Optional[ModelConfig]:
    """The separate draft model's architecture, or None when the target drafts for itself."""
    if not spec_cfg.draft_model and not spec_cfg.draft_preset:
        return None
    dmc = ModelConfig.from_json_file(spec_cfg.draft_model) if spec_cfg.draft_model else \
        get_preset(spec_cfg.draft_preset)
    if dmc.vocab_size != target.vocab_size:
        raise ValueError("draft and target must share the vocabulary")
    return dataclasses.replace(dmc, max_position_embeddings=max(dmc.max_position_embeddings,
                                                               target.max_position_embeddings))


def draft_memory(target: ModelConfig, spec_cfg, dtype_bytes: int, block_size: int) -> Tuple[int, int]:
    """(weight bytes, KV bytes per cache block) the draft adds on the GPU that holds
    it: the draft keeps one KV block per target block (same block tables).  Tensor-
    parallel engines keep an unsharded draft on rank 0."""
    dmc = draft_model_config(target, spec_cfg) if spec_cfg is not None else None
    if dmc is None:
        return 0, 0
    return dmc.num_params() * dtype_bytes, dmc.kv_bytes_per_token(dtype_bytes) * block_size


class SpecDecoder:
    def __init__(self, engine, spec_cfg):
        self.engine = engine
        self.k = spec_cfg.num_speculative_tokens
        self.ngram = getattr(spec_cfg, "method", "draft") == "ngram"
        self.ngram_range = (getattr(spec_cfg, "ngram_max", 4), getattr(spec_cfg, "ngram_min", 1))
        tm = engine.model
        dmc = draft_model_config(tm.cfg, spec_cfg) or dataclasses.replace(tm.cfg)
        self.self_draft = not spec_cfg.draft_model and not spec_cfg.draft_preset
        if self.self_draft:
            self.draft = tm      # sanity mode: the target drafts for itself (acceptance must be 100% when greedy)
        else:
            self.draft = build_model(dmc, dtype=tm.dtype, device=str(tm.device), model_dir=spec_cfg.draft_model,
                                     seed=engine.config.model.seed + 1)
            if tm.device.type == "cuda":
                self.draft.prepare_for_gpu()
        r = engine.runner
        self.runner: ModelRunner = r
        self.drunner = None if self.ngram else ModelRunner(self.draft, num_gpu_blocks=r.num_gpu_blocks, num_cpu_blocks=0,
                                   max_num_seqs=r.max_num_seqs, max_num_batched_tokens=max(
                                       r.max_tokens, r.max_num_seqs * (self.k + 2)),
                                   max_model_len=engine.max_model_len, use_cuda_graph=False)
        # verify forwards need room for S*(k+1) tokens in the target's staging buffers
        need = r.max_num_seqs * (self.k + 1)
        if r.max_tokens < need:
            raise ValueError(f"max_num_batched_tokens must be >= max_num_seqs*(k+1) = {need} for speculation")
        self.draft_computed: Dict[int, int] = {}
        self.stats = {"rounds": 0, "proposed": 0, "accepted": 0, "emitted": 0}

    # ------------------------------------------------------------------ main
    def step(self):
        eng = self.engine
        self._steps = getattr(self, "_steps", 0) + 1
        if self._steps % 256 == 0 and len(self.draft_computed) > len(eng.seq_to_request):
            # sequences of aborted requests never reach the finish path that drops their entry
            self.draft_computed = {k: v for k, v in self.draft_computed.items() if k in eng.seq_to_request}
        so = eng.scheduler.schedule()
        # preempted sequences lose their draft KV (swapped or freed): the draft recomputes it
        for s in so.preempted:
            if not self.self_draft:
                self.draft_computed[s.seq_id] = 0
        if not self.self_draft and so.blocks_to_copy:
            self.drunner.copy_blocks(so.blocks_to_copy)      # the draft's own copy-on-write copies
        if so.is_empty():
            # a step may only move blocks (preemptions with nothing left to run)
            self.runner.apply_block_ops(so)
            return eng._collect_ignored()
        spec_ok = not so.prefills and all(
            s.seq.request.params.top_k <= 0 and s.seq.request.params.top_p >= 1.0 and
            s.seq.request.params.min_p == 0.0 and not s.seq.request.params.needs_host_sampling()
            and not s.seq.request.params.has_penalties() and s.seq.request.params.logprobs is None
            and s.seq.request.params.guided_decoding is None
            and (not self.ngram or s.seq.request.params.is_greedy)
            for s in so.decodes)
        if not spec_ok:
            return self._plain_step(so)
        props = None
        if self.ngram:
            props = self._ngram_proposals([s.seq for s in so.decodes])
            if not props[1].any():
                return self._plain_step(so)
        return self._spec_round(so, props)

    def _ngram_proposals(self, seqs):
        """(int64 [S, k] proposals, int32 [S] how many of each row are real) by prompt lookup."""
        from rusteeze_b200 import _host
        n_max, n_min = self.ngram_range
        props, counts = _host.ngram_propose([s.tokens_np() for s in seqs], self.k, n_max, n_min)
        return torch.from_numpy(props), counts

    def _plain_step(self, so):
        """Normal engine step on the target; the draft processes the same tokens."""
        eng = self.engine
        rows, owners = eng._sample_rows(so)
        self._draft_follow(so)
        t0 = time.monotonic()
        res = eng.runner.execute(so, eng.bm, rows)
        now = time.monotonic()
        eng.stats_counters["steps"] += 1
        touched = eng._apply_results(so, res, owners, now)
        for ss in so.scheduled:
            self.draft_computed[ss.seq.seq_id] = ss.ctx + ss.num_new
        for obs in eng.observers:
            obs(eng, so, now - t0)
        return eng._emit(touched) + eng._collect_ignored()

    def _draft_follow(self, so) -> None:
        if self.self_draft:
            return          # the target's own KV is the draft's KV
        sched = so.scheduled
        if not sched:
            return
        ids = [s.seq.seq_id for s in sched]
        ctx = [s.ctx for s in sched]
        nn = [s.num_new for s in sched]
        toks = np.concatenate([s.seq.tokens_np()[s.ctx:s.ctx + s.num_new] for s in sched])
        self.drunner.forward_arrays(self.engine.bm, ids, ctx, nn, toks, 1, num_decode=0)

    @torch.no_grad()
    def _spec_round(self, so, props=None):
        eng, k, bm = self.engine, self.k, self.engine.bm
        self.runner.apply_block_ops(so)          # the target's swaps and copies of this step
        seqs = [s.seq for s in so.decodes]
        S = len(seqs)
        ids = [s.seq_id for s in seqs]
        cs = [s.num_computed for s in seqs]             # KV exists for positions < c; token at c is new
        t0 = time.monotonic()
        temps = torch.tensor([s.request.params.temperature if not s.request.params.is_greedy else 0.0
                              for s in seqs], dtype=torch.float32)
        if props is not None:
            draft_tokens, n_real = props
            dl = None                  # greedy verification reads no draft distribution
        else:
            draft_tokens, dl = self._draft_proposals(seqs, cs, temps)
            n_real = None
        # ---- one target pass over k+1 positions per sequence
        vt = np.concatenate([np.concatenate([[s.token_ids[c]], draft_tokens[j].numpy()])
                             for j, (s, c) in enumerate(zip(seqs, cs))]).astype(np.int64)
        tlogits = self.runner.forward_arrays(bm, ids, cs, [k + 1] * S, vt, k + 1, num_decode=0)
        seeds = torch.tensor([(s.request.seed + 7919 * s.index) & ((1 << 62) - 1) for s in seqs], dtype=torch.int64)
        offs = torch.tensor([s.num_generated for s in seqs], dtype=torch.int64)
        if tlogits.is_cuda:
            dev = tlogits.device
            out = torch.empty(S, k + 1, dtype=torch.int64, device=dev)
            nacc = torch.empty(S, dtype=torch.int32, device=dev)
            ops.cuda_ext().spec_verify(out, nacc, tlogits.float().contiguous(),
                                       dl.float().contiguous() if dl is not None else None,
                                       draft_tokens.to(dev),
                                       temps.to(dev), seeds.to(dev), offs.to(dev))
            ops.add_launches(1)
            both = torch.cat([out.cpu(), nacc.cpu().long().view(-1, 1)], dim=1)
            out, nacc = both[:, :k + 1], both[:, k + 1]
        else:
            nacc, out = _verify_cpu(tlogits, dl, draft_tokens, temps, seeds, offs)
        now = time.monotonic()
        # ---- apply
        touched, seen = [], set()
        for j, s in enumerate(seqs):
            a = int(nacc[j])
            emitted = [int(x) for x in out[j, :a + 1].tolist()]
            c = cs[j]
            # n-gram rows pad their proposals; only the real ones count
            real = k if n_real is None else int(n_real[j])
            self.stats["proposed"] += real
            self.stats["accepted"] += min(a, real)
            req = s.request
            for tok in emitted:
                s.append_token(tok)
                if req.metrics.first_token_time is None:
                    req.metrics.first_token_time = now
                req.metrics.last_token_time = now
                req.metrics.num_generated = max(req.metrics.num_generated, s.num_generated)
                eng.stats_counters["generation_tokens"] += 1
                self.stats["emitted"] += 1
                try:
                    eng._check_stop(s, tok)
                except Exception as e:  # noqa: BLE001 -- this request's host-side processing only
                    eng._fail_request(req, e)
                if s.is_finished():
                    break
            if not s.is_finished():
                s.num_computed = c + a + 1
                bm.commit(s.seq_id, s.tokens_np(), s.num_computed)
                self.draft_computed[s.seq_id] = c + min(a, k - 1) + 1 if not self.self_draft else s.num_computed
            else:
                self.draft_computed.pop(s.seq_id, None)
            if id(req) not in seen:
                seen.add(id(req))
                touched.append(req)
        self.stats["rounds"] += 1
        eng.stats_counters["steps"] += 1
        for obs in eng.observers:
            obs(eng, so, now - t0)
        return eng._emit(touched)

    def _draft_proposals(self, seqs, cs, temps):
        """k batched draft-model steps: (int64 [S, k] proposals, [S*k, V] draft logits,
        row b*k + j)."""
        k, bm, S = self.k, self.engine.bm, len(seqs)
        ids = [s.seq_id for s in seqs]
        drunner = self.runner if self.self_draft else self.drunner
        dc = [self.draft_computed.get(s.seq_id, s.num_computed) for s in seqs]
        if self.self_draft:
            dc = list(cs)
        n1 = [c - d + 1 for c, d in zip(cs, dc)]
        if not self.self_draft and sum(n1) > drunner.max_tokens:
            # a long catch-up (a preempted sequence recomputes its draft KV): feed the tokens
            # before each sequence's current one in chunks that fit the draft runner
            self._draft_catch_up(seqs, dc, cs, drunner)
            dc = list(cs)
            n1 = [1] * S
        toks = np.concatenate([s.tokens_np()[d:c + 1] for s, d, c in zip(seqs, dc, cs)])
        draft_tokens = torch.empty(S, k, dtype=torch.long)
        draft_logits = []
        cur = None
        for i in range(k):
            if i == 0:
                logits = drunner.forward_arrays(bm, ids, dc, n1, toks, 1, num_decode=0)
            else:
                logits = drunner.forward_arrays(bm, ids, [c + i for c in cs], [1] * S, cur, 1, num_decode=S)
            draft_logits.append(logits)
            nxt = self._propose(logits, temps, seqs, i)
            draft_tokens[:, i] = nxt
            cur = nxt.numpy()
        return draft_tokens, torch.stack(draft_logits, dim=1).reshape(S * k, -1)

    def _draft_catch_up(self, seqs, dc, cs, drunner) -> None:
        """Draft KV for positions [dc[i], cs[i]) of every sequence, in batches of at most
        the draft runner's token capacity (logits are not needed)."""
        cap = drunner.max_tokens
        todo = [(s, d, c) for s, d, c in zip(seqs, dc, cs) if c > d]
        while todo:
            ids, ctx, nn, parts, used, rest = [], [], [], [], 0, []
            for s, d, c in todo:
                take = min(c - d, cap - used)
                if take <= 0 or len(ids) == drunner.max_num_seqs:
                    rest.append((s, d, c))
                    continue
                ids.append(s.seq_id)
                ctx.append(d)
                nn.append(take)
                parts.append(s.tokens_np()[d:d + take])
                used += take
                if d + take < c:
                    rest.append((s, d + take, c))
            drunner.forward_arrays(self.engine.bm, ids, ctx, nn, np.concatenate(parts), 1, num_decode=0)
            todo = rest

    def _propose(self, logits: torch.Tensor, temps: torch.Tensor, seqs, i: int) -> torch.Tensor:
        """Greedy argmax, or a temperature sample (Gumbel-max) per row."""
        lg = logits.float()
        if bool((temps <= 0).all()):
            return lg.argmax(-1).cpu()
        g = torch.Generator(device=lg.device)
        g.manual_seed(int(seqs[0].request.seed) + 104729 * (seqs[0].num_generated + i))
        u = torch.rand(lg.shape, generator=g, device=lg.device).clamp_(1e-12, 1.0)
        t = temps.to(lg.device).clamp_min(1e-5).unsqueeze(1)
        keys = torch.where(temps.to(lg.device).unsqueeze(1) > 0, lg / t - torch.log(-torch.log(u)), lg)
        return keys.argmax(-1).cpu()

    def acceptance_rate(self) -> float:
        return self.stats["accepted"] / max(1, self.stats["proposed"])
