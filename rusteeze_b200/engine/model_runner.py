"""Per-GPU model runner: KV cache, batch staging, CUDA graphs, sampling.

The reference's worker (crates/rusteeze-engine/src/worker.rs:56-164) keeps a
preallocated logits buffer and calls an injected model closure.  Here the
runner owns everything between a scheduler decision and sampled tokens:

  * KV cache: one device tensor [num_blocks, L, 2, Hkv, 16, D].  A block holds
    the K and V of 16 tokens for every layer contiguously, so a swap or a
    copy-on-write copy is one contiguous transfer per block, while each
    (block, layer, k|v, head) tile the attention kernels read is a
    contiguous 4 KiB run (Hkv=1 slice: 16 x 128 bf16).
  * Swap space: the same layout in pinned host memory (`swap_space` GiB).
  * Batch staging: the C++ batch builder writes ids/positions/slots/
    cu-seqlens/block tables into pinned host buffers, which are copied to
    static device buffers with one async H2D each.
  * CUDA graphs: pure-decode steps are replayed from graphs captured per
    batch-size bucket (1, 2, 4, 8, 16, 24, 32, ... max_num_seqs); the decode
    attention's split count is fixed per bucket and the split range is
    derived from the live sequence lengths inside the kernel.
  * Sampling happens on the device; only token ids (and logprobs if asked)
    come back.
"""
from __future__ import annotations

import math
import time
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from rusteeze_b200.engine.sampler import SampleRow, Sampler, SampleResult
from rusteeze_b200.engine.scheduler import SchedulerOutput
from rusteeze_b200.models.decoder import AttentionMetadata, DecoderLM
from rusteeze_b200.ops import BLOCK_SIZE
from rusteeze_b200.ops import reference as ref
from rusteeze_b200.utils.op_timer import OP_TIMER

_ZERO1 = np.zeros(1, dtype=np.int64)

NUM_SMS_B200 = 148


def decode_graph_buckets(max_seqs: int) -> List[int]:
    b = [1, 2, 4, 8, 16]
    x = 24
    while x < max_seqs:
        b.append(x)
        x += 8 if x < 64 else 16 if x < 128 else 32
    b.append(max_seqs)
    return sorted(set(v for v in b if v <= max_seqs))


def choose_num_splits(batch: int, num_kv_heads: int, max_blocks: int, num_sms: int = NUM_SMS_B200,
                      warps_per_sm: int = 8) -> int:
    """Split-KV factor for the decode kernel, whose work item is one warp per
    (sequence, kv head, split): aim for about two items per resident warp so
    the last wave is short."""
    items = batch * num_kv_heads
    target = 2 * num_sms * warps_per_sm
    if items >= target:
        return 1
    s = math.ceil(target / items)
    return max(1, min(s, max_blocks, 64))


def decode_workspace_floats(max_seqs: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                            max_blocks: int) -> int:
    """Largest split-KV partial buffer any batch size up to max_seqs needs."""
    need = 0
    for b in range(1, max_seqs + 1):
        s = choose_num_splits(b, num_kv_heads, max_blocks)
        if s > 1:
            need = max(need, b * num_q_heads * s * (head_dim + 2))
    return max(need, 1)


class ModelRunner:
    supports_async = True     # launch / finish: the engine may pipeline steps over this runner

    def __init__(self, model: DecoderLM, *, num_gpu_blocks: int, num_cpu_blocks: int,
                 max_num_seqs: int, max_num_batched_tokens: int, max_model_len: int,
                 kv_dtype=None, use_cuda_graph: bool = True, seed: int = 0):
        self.model = model
        self.cfg = model.cfg
        self.device = model.device
        self.is_cuda = self.device.type == "cuda"
        self.max_num_seqs = max_num_seqs
        self.max_tokens = max(max_num_batched_tokens, max_num_seqs)
        self.max_blocks = (max_model_len + BLOCK_SIZE - 1) // BLOCK_SIZE
        self.kv_dtype = kv_dtype or model.dtype
        L, D, hkv = self.cfg.num_hidden_layers, self.cfg.head_dim, model.hkv
        self.num_gpu_blocks = num_gpu_blocks
        # fp8 caches are allocated and moved as bytes (block copies, swaps) and viewed as
        # their float8 dtype by the attention ops
        store = torch.uint8 if ref.is_fp8(self.kv_dtype) else self.kv_dtype
        self.kv_cache = torch.zeros(num_gpu_blocks, L, 2, hkv, BLOCK_SIZE, D, dtype=store,
                                    device=self.device).view(self.kv_dtype)
        self.kv_layers = [(self.kv_cache[:, l, 0], self.kv_cache[:, l, 1]) for l in range(L)]
        self.cpu_cache = None
        if num_cpu_blocks > 0:
            self.cpu_cache = torch.zeros(num_cpu_blocks, L, 2, hkv, BLOCK_SIZE, D, dtype=store,
                                         pin_memory=self.is_cuda).view(self.kv_dtype)
        pin = self.is_cuda
        T, S, MB = self.max_tokens, max_num_seqs, self.max_blocks
        # two sets of pinned staging buffers, alternated per step: with
        # asynchronous scheduling the next step is prepared while the previous
        # step's host->device copies may still be queued behind the GPU
        self._host_sets = [self._alloc_host(T, S, MB, pin) for _ in range(2)]
        self._host_k = 0
        self._bind_host(0)
        dev = self.device
        self.d_input_ids = torch.zeros(T, dtype=torch.int64, device=dev)
        self.d_positions = torch.zeros(T, dtype=torch.int64, device=dev)
        self.d_slots = torch.full((T,), -1, dtype=torch.int64, device=dev)
        self.d_qsl = torch.zeros(S + 1, dtype=torch.int32, device=dev)
        self.d_seq_lens = torch.zeros(S, dtype=torch.int32, device=dev)
        self.d_block_tables = torch.zeros(S, MB, dtype=torch.int32, device=dev)
        self.d_logits_idx = torch.zeros(T, dtype=torch.int64, device=dev)
        self.decode_ws = (torch.empty(decode_workspace_floats(S, model.hq, hkv, D, self.max_blocks),
                                      dtype=torch.float32, device=dev) if self.is_cuda else None)
        self.sampler = Sampler(self.cfg.vocab_size)
        self.use_cuda_graph = use_cuda_graph and self.is_cuda
        self.graphs: Dict[int, Tuple[torch.cuda.CUDAGraph, torch.Tensor]] = {}
        self.graph_pool = None
        self.seed = seed
        self.graph_launches: Dict[int, int] = {}
        self.h2d_bytes = 0      # host->device bytes staged per step (cumulative)
        self.phase_s: Dict[str, float] = {"prepare": 0.0, "enqueue": 0.0, "sample_wait": 0.0}
        self.d2h_bytes = 0      # device->host bytes read back (cumulative)

    @staticmethod
    def _alloc_host(T: int, S: int, MB: int, pin: bool) -> Dict[str, torch.Tensor]:
        return {"h_input_ids": torch.zeros(T, dtype=torch.int64, pin_memory=pin),
                "h_positions": torch.zeros(T, dtype=torch.int64, pin_memory=pin),
                "h_slots": torch.zeros(T, dtype=torch.int64, pin_memory=pin),
                "h_qsl": torch.zeros(S + 1, dtype=torch.int32, pin_memory=pin),
                "h_seq_lens": torch.zeros(S, dtype=torch.int32, pin_memory=pin),
                "h_block_tables": torch.zeros(S, MB, dtype=torch.int32, pin_memory=pin),
                "h_logits_idx": torch.zeros(T, dtype=torch.int64, pin_memory=pin),
                "h_sample_idx": torch.zeros(T, dtype=torch.int64, pin_memory=pin),
                "h_pend": torch.zeros(2 * S, dtype=torch.int64, pin_memory=pin)}

    def _bind_host(self, k: int) -> None:
        for name, t in self._host_sets[k].items():
            setattr(self, name, t)
        self.h_logits_idx_np = self.h_logits_idx.numpy()
        self.h_seq_lens_np = self.h_seq_lens.numpy()

    def prefill_kv_blocks(self, nd: int, S: int) -> int:
        """KV blocks of sequences [nd, S) of the staged batch (host lengths)."""
        if S <= nd or not ref.is_fp8(self.kv_dtype):
            return 0
        return int(((self.h_seq_lens_np[nd:S].astype(np.int64) + BLOCK_SIZE - 1) // BLOCK_SIZE).sum())

    def _flip_host(self) -> None:
        self._host_k ^= 1
        self._bind_host(self._host_k)

    # ------------------------------------------------------------------ cache ops
    @torch.no_grad()
    def copy_blocks(self, pairs: List[Tuple[int, int]]) -> None:
        if not pairs:
            return
        src = torch.tensor([p[0] for p in pairs], dtype=torch.long, pin_memory=self.is_cuda).to(
            self.device, non_blocking=True)
        dst = torch.tensor([p[1] for p in pairs], dtype=torch.long, pin_memory=self.is_cuda).to(
            self.device, non_blocking=True)
        kv = self.kv_cache.view(torch.uint8) if ref.is_fp8(self.kv_dtype) else self.kv_cache
        kv.index_copy_(0, dst, kv.index_select(0, src))

    @torch.no_grad()
    def swap_out(self, pairs: List[Tuple[int, int]]) -> None:
        for g, c in pairs:   # one contiguous D2H per block
            self.cpu_cache[c].copy_(self.kv_cache[g], non_blocking=True)

    @torch.no_grad()
    def swap_in(self, pairs: List[Tuple[int, int]]) -> None:
        for c, g in pairs:
            self.kv_cache[g].copy_(self.cpu_cache[c], non_blocking=True)

    # ------------------------------------------------------------------ batch prep
    def prepare(self, so: SchedulerOutput, bm,
                prev_tokens: Optional[torch.Tensor] = None) -> Tuple[AttentionMetadata, int, int, List[int]]:
        """Builds the step's batch.  With asynchronous scheduling a decode
        whose input token is still on the device (ScheduledSeq.pend_row >= 0)
        gets a placeholder here and is filled from `prev_tokens` (the previous
        step's sampled ids) by a device-side scatter after the copies."""
        self._flip_host()
        sched = so.scheduled
        S = len(sched)
        seq_ids = np.fromiter((s.seq.seq_id for s in sched), dtype=np.int64, count=S)
        ctx = np.fromiter((s.ctx for s in sched), dtype=np.int64, count=S)
        n_new = np.fromiter((s.num_new for s in sched), dtype=np.int64, count=S)
        pend_dst: List[int] = []
        pend_src: List[int] = []
        if S:
            parts = []
            off = 0
            for s in sched:
                if s.pend_row >= 0:
                    pend_dst.append(off)
                    pend_src.append(s.pend_row)
                    parts.append(_ZERO1)
                else:
                    parts.append(s.seq.tokens_np()[s.ctx:s.ctx + s.num_new])
                off += s.num_new
            toks = np.concatenate(parts)
        else:
            toks = np.zeros(0, dtype=np.int64)
        self.last_pend = (pend_dst, pend_src)     # the scatter a tensor-parallel worker repeats
        self._check_capacity(S, int(n_new.sum()))
        T = bm.build_batch(seq_ids, ctx, n_new, toks, self.h_input_ids.data_ptr(),
                           self.h_positions.data_ptr(), self.h_slots.data_ptr(), self.h_qsl.data_ptr(),
                           self.h_seq_lens.data_ptr(), self.h_block_tables.data_ptr(),
                           self.h_logits_idx.data_ptr(), self.max_blocks, 1)
        # rows to sample: last token of sequences with sample=True, repeated num_samples times
        lidx = self.h_logits_idx_np
        sample_rows: List[int] = []
        for i, s in enumerate(sched):
            if s.sample:
                li = int(lidx[i])
                sample_rows.extend([li] * s.num_samples)
        nd = len(so.decodes)
        max_q = max((s.num_new for s in so.prefills), default=1)
        max_s = int(self.h_seq_lens_np[:S].max()) if S else 0
        nb = non_blocking = self.is_cuda
        self.h2d_bytes += 3 * 8 * T + 4 * (S + 1) + 4 * S + 4 * S * self.max_blocks
        self.d_input_ids[:T].copy_(self.h_input_ids[:T], non_blocking=nb)
        self.d_positions[:T].copy_(self.h_positions[:T], non_blocking=nb)
        self.d_slots[:T].copy_(self.h_slots[:T], non_blocking=nb)
        self.d_qsl[:S + 1].copy_(self.h_qsl[:S + 1], non_blocking=nb)
        self.d_seq_lens[:S].copy_(self.h_seq_lens[:S], non_blocking=nb)
        self.d_block_tables[:S].copy_(self.h_block_tables[:S], non_blocking=non_blocking)
        if pend_dst:
            if prev_tokens is None:
                raise RuntimeError("pending decode input without the previous step's samples")
            P = len(pend_dst)
            hp = self.h_pend[:2 * P]              # [dst | src], a contiguous prefix of a pinned buffer
            hp.copy_(torch.from_numpy(np.asarray(pend_dst + pend_src, dtype=np.int64)))
            dp = hp.to(self.device, non_blocking=nb)
            self.d_input_ids.index_copy_(0, dp[:P], prev_tokens.index_select(0, dp[P:]))
            self.h2d_bytes += 16 * P
        meta = AttentionMetadata(
            num_seqs=S, num_tokens=T, num_decode_seqs=nd, query_start_loc=self.d_qsl[:S + 1],
            seq_lens=self.d_seq_lens[:S], block_tables=self.d_block_tables[:S],
            slot_mapping=self.d_slots[:T], max_query_len=max_q, max_seq_len=max_s,
            decode_num_splits=choose_num_splits(max(nd, 1), self.model.hkv, self.max_blocks),
            decode_workspace=self.decode_ws, prefill_kv_blocks=self.prefill_kv_blocks(nd, S))
        if not self.is_cuda:
            # host oracle path reads the metadata on the host
            meta.query_start_loc = self.h_qsl[:S + 1].clone()
            meta.seq_lens = self.h_seq_lens[:S].clone()
            meta.block_tables = self.h_block_tables[:S].clone()
        return meta, T, S, sample_rows

    @torch.no_grad()
    def forward_arrays(self, bm, seq_ids, ctx, n_new, toks, logits_per_seq: int,
                       num_decode: int = 0, hidden: bool = False) -> torch.Tensor:
        """Eager forward of an explicit token batch (speculative decoding, prompt scoring,
        embeddings): sequence i gets n_new[i] tokens at positions ctx[i].., and the logits
        (or, with `hidden`, the final normalised hidden states) of its last
        `logits_per_seq` tokens are returned in sequence order."""
        meta, T, S = self.stage_arrays(bm, seq_ids, ctx, n_new, toks, logits_per_seq, num_decode)
        return self.forward_staged(meta, T, S * logits_per_seq, hidden=hidden)

    def forward_staged(self, meta, T: int, n_rows: int, hidden: bool = False) -> torch.Tensor:
        """Forward of the staged batch; logits (or hidden states) of the rows
        h_logits_idx[:n_rows].  A tensor-parallel rank computes the logits even when it
        returns hidden states: the LM head's all-gather is a collective that every rank
        joins."""
        h = self.model(self.d_input_ids[:T], self.d_positions[:T], meta, self.kv_layers)
        idx = self.h_logits_idx[:n_rows].to(h.device, non_blocking=self.is_cuda)
        hs = h.index_select(0, idx)
        if hidden and self.model.tp.size == 1:
            return hs
        logits = self.model.compute_logits(hs)
        return hs if hidden else logits

    def stage_arrays(self, bm, seq_ids, ctx, n_new, toks, logits_per_seq: int, num_decode: int = 0):
        """Builds and uploads the batch of `forward_arrays` (block tables from `bm`);
        returns (metadata, T, S)."""
        S = len(seq_ids)
        self._check_capacity(S, int(np.sum(n_new)) if S else 0)
        self._flip_host()
        T = bm.build_batch(np.asarray(seq_ids, dtype=np.int64), np.asarray(ctx, dtype=np.int64),
                           np.asarray(n_new, dtype=np.int64), np.asarray(toks, dtype=np.int64),
                           self.h_input_ids.data_ptr(), self.h_positions.data_ptr(), self.h_slots.data_ptr(),
                           self.h_qsl.data_ptr(), self.h_seq_lens.data_ptr(), self.h_block_tables.data_ptr(),
                           self.h_logits_idx.data_ptr(), self.max_blocks, logits_per_seq)
        nb = self.is_cuda
        self.d_input_ids[:T].copy_(self.h_input_ids[:T], non_blocking=nb)
        self.d_positions[:T].copy_(self.h_positions[:T], non_blocking=nb)
        self.d_slots[:T].copy_(self.h_slots[:T], non_blocking=nb)
        self.d_qsl[:S + 1].copy_(self.h_qsl[:S + 1], non_blocking=nb)
        self.d_seq_lens[:S].copy_(self.h_seq_lens[:S], non_blocking=nb)
        self.d_block_tables[:S].copy_(self.h_block_tables[:S], non_blocking=nb)
        self.h2d_bytes += 3 * 8 * T + 8 * S + 4 * S * self.max_blocks
        meta = AttentionMetadata(
            num_seqs=S, num_tokens=T, num_decode_seqs=num_decode, query_start_loc=self.d_qsl[:S + 1],
            seq_lens=self.d_seq_lens[:S], block_tables=self.d_block_tables[:S], slot_mapping=self.d_slots[:T],
            max_query_len=int(max(n_new)) if S else 1, max_seq_len=int(self.h_seq_lens[:S].max()) if S else 0,
            decode_num_splits=choose_num_splits(max(num_decode, 1), self.model.hkv, self.max_blocks),
            decode_workspace=self.decode_ws, prefill_kv_blocks=self.prefill_kv_blocks(num_decode, S))
        if not self.is_cuda:
            meta.query_start_loc = self.h_qsl[:S + 1].clone()
            meta.seq_lens = self.h_seq_lens[:S].clone()
            meta.block_tables = self.h_block_tables[:S].clone()
        return meta, T, S

    # ------------------------------------------------------------------ graphs
    def _graph_bucket(self, n: int) -> Optional[int]:
        for b in sorted(self.graphs):
            if b >= n:
                return b
        return None

    def release_graphs(self) -> None:
        """Drops the captured graphs and their memory pool.  Graphs that contain
        NCCL collectives must be released before the process group is
        destroyed, or the teardown waits on them forever."""
        self.graphs = {}
        self.graph_pool = None
        import gc
        gc.collect()
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
            torch.cuda.empty_cache()

    @torch.no_grad()
    def capture_graphs(self, buckets: Optional[List[int]] = None) -> None:
        """Captures decode-only forward + LM head for each batch bucket."""
        if not self.use_cuda_graph:
            return
        buckets = buckets or decode_graph_buckets(self.max_num_seqs)
        self.graph_pool = torch.cuda.graph_pool_handle()
        stream = torch.cuda.Stream()
        for B in sorted(buckets, reverse=True):
            meta = self._graph_meta(B)
            self.d_slots[:B].fill_(-1)
            self.d_seq_lens[:B].fill_(0)
            self.d_block_tables[:B].zero_()
            self.d_input_ids[:B].zero_()
            self.d_positions[:B].zero_()
            # the side stream must see the buffer initialisation above
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                for _ in range(2):     # warm-up outside capture
                    self._decode_forward(B, meta)
            torch.cuda.current_stream().wait_stream(stream)
            g = torch.cuda.CUDAGraph()
            from rusteeze_b200 import ops as _ops
            n0 = _ops.launch_count()
            with torch.cuda.graph(g, pool=self.graph_pool, stream=stream):
                out = self._decode_forward(B, meta)
            self.graph_launches[B] = _ops.launch_count() - n0
            self.graphs[B] = (g, out, meta)
        torch.cuda.synchronize()

    def _graph_meta(self, B: int) -> AttentionMetadata:
        return AttentionMetadata(
            num_seqs=B, num_tokens=B, num_decode_seqs=B, query_start_loc=self.d_qsl[:B + 1],
            seq_lens=self.d_seq_lens[:B], block_tables=self.d_block_tables[:B],
            slot_mapping=self.d_slots[:B], max_query_len=1, max_seq_len=self.max_blocks * BLOCK_SIZE,
            decode_num_splits=choose_num_splits(B, self.model.hkv, self.max_blocks),
            decode_workspace=self.decode_ws)

    def _decode_forward(self, B: int, meta: AttentionMetadata) -> torch.Tensor:
        h = self.model(self.d_input_ids[:B], self.d_positions[:B], meta, self.kv_layers)
        return self.model.compute_logits(h)

    # ------------------------------------------------------------------ execute
    @torch.no_grad()
    def _check_capacity(self, S: int, T: int) -> None:
        """The batch builder writes into the fixed-size staging buffers: refuse a batch
        that does not fit them instead of writing past their ends."""
        if S > self.max_num_seqs or T > self.max_tokens:
            raise ValueError(f"batch of {S} sequences / {T} tokens exceeds this runner's staging capacity "
                             f"({self.max_num_seqs} sequences / {self.max_tokens} tokens)")

    def apply_block_ops(self, so: SchedulerOutput) -> None:
        """The step's KV block moves: swap-outs first (their GPU blocks may be handed to
        swap-ins and copies of the same step), then swap-ins, then copy-on-write copies."""
        if so.blocks_to_swap_out:
            self.swap_out(so.blocks_to_swap_out)
        if so.blocks_to_swap_in:
            self.swap_in(so.blocks_to_swap_in)
        if so.blocks_to_copy:
            self.copy_blocks(so.blocks_to_copy)

    # ------------------------------------------------------------------ asynchronous steps
    @torch.no_grad()
    def launch(self, so: SchedulerOutput, bm, rows: List[SampleRow], prev_tokens: Optional[torch.Tensor]):
        """Enqueues a whole step (copies, forward, sampling, result readback)
        without waiting for the GPU; `finish` returns its SampleResult."""
        self.apply_block_ops(so)
        t0 = time.perf_counter()
        meta, T, S, sample_rows = self.prepare(so, bm, prev_tokens)
        t1 = time.perf_counter()
        logits = self.forward_logits(meta, T, S, sample_rows, pure_decode=not so.prefills)
        t2 = time.perf_counter()
        handle = self.sampler.launch(logits, rows)
        ph = self.phase_s
        ph["prepare"] += t1 - t0
        ph["enqueue"] += time.perf_counter() - t1
        self.h2d_bytes += self.sampler.last_h2d_bytes
        return handle

    def finish(self, handle) -> SampleResult:
        t0 = time.perf_counter()
        res = self.sampler.finish(handle)
        self.phase_s["sample_wait"] += time.perf_counter() - t0
        self.d2h_bytes += self.sampler.last_d2h_bytes
        return res

    def execute(self, so: SchedulerOutput, bm, rows: List[SampleRow]) -> SampleResult:
        self.apply_block_ops(so)
        t0 = time.perf_counter()
        meta, T, S, sample_rows = self.prepare(so, bm)
        t1 = time.perf_counter()
        logits = self.forward_logits(meta, T, S, sample_rows, pure_decode=not so.prefills)
        t2 = time.perf_counter()
        res = self.sampler.sample(logits, rows)
        t3 = time.perf_counter()
        # host seconds: batch build, forward enqueue, sampling (includes the wait for the GPU)
        ph = self.phase_s
        ph["prepare"] += t1 - t0
        ph["enqueue"] += t2 - t1
        ph["sample_wait"] += t3 - t2
        self.h2d_bytes += self.sampler.last_h2d_bytes
        self.d2h_bytes += self.sampler.last_d2h_bytes
        return res

    def forward_logits(self, meta: AttentionMetadata, T: int, S: int, sample_rows: List[int],
                       pure_decode: bool) -> torch.Tensor:
        B = self._graph_bucket(S) if (pure_decode and self.graphs and T == S) else None
        if B is not None:
            if B > S:   # padded rows: no KV write, empty context
                self.d_slots[S:B].fill_(-1)
                self.d_seq_lens[S:B].fill_(0)
                self.d_input_ids[S:B].fill_(0)
                self.d_positions[S:B].fill_(0)
            g, out, _ = self.graphs[B]
            with OP_TIMER.section("decode_graph"):
                g.replay()
            from rusteeze_b200 import ops as _ops
            _ops.add_launches(self.graph_launches.get(B, 0))
            if len(sample_rows) == S and sample_rows == list(range(S)):
                return out[:S]                   # every row sampled once, in order: a view
            return out.index_select(0, self._sample_index(sample_rows))
        h = self.model(self.d_input_ids[:T], self.d_positions[:T], meta, self.kv_layers)
        hs = h.index_select(0, self._sample_index(sample_rows))
        return self.model.compute_logits(hs)

    def _sample_index(self, sample_rows: List[int]) -> torch.Tensor:
        n = len(sample_rows)
        hi = self.h_sample_idx[:n]
        hi.copy_(torch.from_numpy(np.asarray(sample_rows, dtype=np.int64)))
        return hi.to(self.device, non_blocking=self.is_cuda)
