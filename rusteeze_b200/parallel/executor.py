"""Tensor-parallel execution: rank 0 schedules, every rank runs the forward.

Rank 0 owns the engine (scheduler, block manager, sampler, API).  For each
step it packs the batch plan -- the staged input arrays (token ids,
positions, slot mapping, cu-seqlens, sequence lengths, block tables),
sample rows, and the swap / copy-on-write block lists -- and publishes it
on a shared-memory broadcast ring (C++ `ShmRing`, no collective and no
device sync on the control path).  Worker ranks (one process per GPU)
consume the plan, stage it into their own pinned buffers, and run the same
forward on their weight shard; the model's collectives (NCCL or the fused
peer-memory kernels) keep them in lock step.  Only rank 0 samples.

Failure handling: every ring wait is bounded; a worker that sees no plan
within `idle_timeout_s` checks the ring's closed flag and rank 0's
liveness, and the process group's timeout turns a dead rank into an error
on the survivors (the engine then reports unhealthy).
"""
from __future__ import annotations

import logging
import pickle
import time
from typing import Optional, Tuple

import torch

from rusteeze_b200.engine.model_runner import ModelRunner
from rusteeze_b200.engine.sampler import SampleResult

log = logging.getLogger("rusteeze.tp")

MSG_STEP, MSG_STOP = 1, 2


def _ring_name(tag: str) -> str:
    return f"/rz_plan_{tag}"


class PlanChannel:
    def __init__(self, tag: str, rank: int, world: int, slot_bytes: int = 8 << 20, create: Optional[bool] = None):
        from rusteeze_b200.engine.block_manager import host_ext
        H = host_ext()
        self.rank, self.world = rank, world
        create = (rank == 0) if create is None else create
        self.ring = H.ShmRing(_ring_name(tag), create, 4, slot_bytes, max(0, world - 1))

    def publish(self, kind: int, payload) -> None:
        data = pickle.dumps((kind, payload), protocol=pickle.HIGHEST_PROTOCOL)
        if not self.ring.publish(data, 60.0):
            raise TimeoutError("tensor-parallel worker did not consume the previous plan within 60 s")

    def consume(self, timeout_s: float = 1.0):
        b = self.ring.consume(self.rank - 1, timeout_s)
        if b is None:
            return None
        return pickle.loads(b)

    def close(self) -> None:
        self.ring.close()


class TPExecutor:
    """Drop-in for ModelRunner on rank 0 (`LLMEngine(executor=...)`).

    Pipelined steps (`launch` / `finish`, on with `engine.async_scheduling`): the next step's plan is
    published before the previous step's tokens are read back.  Decode inputs still on
    the device are scattered from the previous step's sample tensor, which rank 0
    broadcasts to the workers (device to device, one small collective ordered before the
    step's forward); the plan carries the scatter lists."""

    supports_async = True

    def __init__(self, runner: ModelRunner, channel: PlanChannel, liveness=None):
        self.runner = runner
        self.ch = channel
        # callable -> list of dead worker ranks (the launcher watches its child processes);
        # checked before every plan so a dead rank is reported instead of stalling a collective
        self.liveness = liveness
        self._tstate: dict = {}
        self.broadcast_steps = 0     # pipelined steps whose decode inputs came from the previous sample

    def __getattr__(self, k):
        return getattr(self.runner, k)

    def _check_workers(self) -> None:
        if self.liveness is None:
            return
        dead = self.liveness()
        if dead:
            from rusteeze_b200.core.errors import DistributedError
            raise DistributedError(f"tensor-parallel worker rank(s) {dead} exited; the engine must be restarted")

    def capture_graphs(self, buckets=None) -> None:
        self._check_workers()
        self.ch.publish(MSG_STEP, {"capture": list(buckets) if buckets is not None else None})
        self.runner.capture_graphs(buckets)

    @torch.no_grad()
    def execute(self, so, bm, rows) -> SampleResult:
        self._check_workers()
        r = self.runner
        meta, T, S, sample_rows = r.prepare(so, bm)
        plan = {"pure": not so.prefills, "rows": sample_rows, "copy": so.blocks_to_copy,
                "sin": so.blocks_to_swap_in, "sout": so.blocks_to_swap_out, **_staged_plan(r, meta, T, S)}
        self.ch.publish(MSG_STEP, plan)
        if so.blocks_to_swap_out:
            r.swap_out(so.blocks_to_swap_out)
        if so.blocks_to_swap_in:
            r.swap_in(so.blocks_to_swap_in)
        if so.blocks_to_copy:
            r.copy_blocks(so.blocks_to_copy)
        logits = r.forward_logits(meta, T, S, sample_rows, pure_decode=not so.prefills)
        res = r.sampler.sample(logits, rows)
        r.h2d_bytes += r.sampler.last_h2d_bytes
        r.d2h_bytes += r.sampler.last_d2h_bytes
        return res

    @torch.no_grad()
    def launch(self, so, bm, rows, prev_tokens):
        """Enqueues a step on every rank without waiting for the previous one's tokens."""
        import torch.distributed as dist
        self._check_workers()
        r = self.runner
        if so.blocks_to_swap_out:
            r.swap_out(so.blocks_to_swap_out)
        if so.blocks_to_swap_in:
            r.swap_in(so.blocks_to_swap_in)
        if so.blocks_to_copy:
            r.copy_blocks(so.blocks_to_copy)
        meta, T, S, sample_rows = r.prepare(so, bm, prev_tokens)
        pend_dst, pend_src = r.last_pend
        nb = int(prev_tokens.numel()) if pend_dst else 0
        plan = {"pure": not so.prefills, "rows": sample_rows, "copy": so.blocks_to_copy,
                "sin": so.blocks_to_swap_in, "sout": so.blocks_to_swap_out, "bcast": nb,
                "pend": (list(pend_dst), list(pend_src)), **_staged_plan(r, meta, T, S)}
        self.ch.publish(MSG_STEP, plan)
        if nb:
            dist.broadcast(prev_tokens.contiguous(), src=0)
            self.broadcast_steps += 1
        logits = r.forward_logits(meta, T, S, sample_rows, pure_decode=not so.prefills)
        handle = r.sampler.launch(logits, rows)
        r.h2d_bytes += r.sampler.last_h2d_bytes
        return handle

    def finish(self, handle) -> SampleResult:
        return self.runner.finish(handle)

    def apply_block_ops(self, so) -> None:
        """A step's swap / copy-on-write block moves outside a step plan (speculative
        rounds run their forwards as explicit batches): every rank moves its own KV shard."""
        if so.blocks_to_swap_out or so.blocks_to_swap_in or so.blocks_to_copy:
            self._check_workers()
            self.ch.publish(MSG_STEP, {"blockops": (so.blocks_to_swap_out, so.blocks_to_swap_in, so.blocks_to_copy)})
            self.runner.apply_block_ops(so)

    @torch.no_grad()
    def forward_arrays(self, bm, seq_ids, ctx, n_new, toks, logits_per_seq: int,
                       num_decode: int = 0, hidden: bool = False) -> torch.Tensor:
        """Speculative-decoding forwards (draft on the target, verify): rank 0 stages
        the explicit token batch, the plan carries its arrays and logits rows, and
        every rank runs the same forward on its shard."""
        self._check_workers()
        r = self.runner
        meta, T, S = r.stage_arrays(bm, seq_ids, ctx, n_new, toks, logits_per_seq, num_decode)
        n_rows = S * logits_per_seq
        self.ch.publish(MSG_STEP, {"arrays": n_rows, **_staged_plan(r, meta, T, S)})
        return r.forward_staged(meta, T, n_rows, hidden=hidden)

    def timer(self, kind: str):
        """Device-timed window over every rank: "start" marks it on each rank's stream,
        "stop" returns its length in ms, the MAX over ranks (one all-reduce that the
        workers join when they consume the stop message, after their last step)."""
        self._check_workers()
        self.ch.publish(MSG_STEP, {"timer": kind})
        return _timer_mark(self.runner, kind, self._tstate)

    def shutdown(self) -> None:
        try:
            self.ch.publish(MSG_STOP, None)
        finally:
            self.ch.close()


def _staged_plan(r: ModelRunner, meta, T: int, S: int) -> dict:
    """The staged host arrays of a batch (rank 0), as the workers' `stage_plan` reads them."""
    MB = int(max(1, (int(r.h_seq_lens[:S].max()) + 15) // 16)) if S else 1
    return {
        "T": T, "S": S, "nd": meta.num_decode_seqs, "maxq": meta.max_query_len, "maxs": meta.max_seq_len,
        "mb": MB, "ids": r.h_input_ids[:T].numpy().copy(), "pos": r.h_positions[:T].numpy().copy(),
        "slots": r.h_slots[:T].numpy().copy(), "qsl": r.h_qsl[:S + 1].numpy().copy(),
        "sl": r.h_seq_lens[:S].numpy().copy(), "bt": r.h_block_tables[:S, :MB].numpy().copy(),
        "lidx": r.h_logits_idx[:T].numpy().copy(),
    }


def _timer_mark(runner: ModelRunner, kind: str, state: dict):
    """One rank's side of `TPExecutor.timer`: CUDA events on the runner's stream (host
    clock on CPU ranks); "stop" all-reduces the elapsed ms with MAX over ranks.
    "ops_start" / "ops_stop" switch the per-section op timer on every rank; "ops_stop"
    returns ms per section, the MAX over ranks."""
    import torch.distributed as dist
    from rusteeze_b200.utils.op_timer import OP_TIMER, SECTIONS
    cuda = runner.is_cuda
    if kind == "ops_start":
        OP_TIMER.start()
        return None
    if kind == "ops_stop":
        OP_TIMER.stop()
        rep = OP_TIMER.report() if cuda else {}
        t = torch.tensor([rep.get(k, 0.0) for k in SECTIONS], dtype=torch.float64,
                         device=torch.cuda.current_device() if cuda else "cpu")
        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return dict(zip(SECTIONS, t.tolist()))
    if kind == "start":
        if cuda:
            state["ev0"] = torch.cuda.Event(enable_timing=True)
            state["ev0"].record()
        else:
            state["t0"] = time.perf_counter()
        return None
    if cuda:
        ev1 = torch.cuda.Event(enable_timing=True)
        ev1.record()
        torch.cuda.synchronize()
        ms = state["ev0"].elapsed_time(ev1)
        t = torch.tensor([ms], dtype=torch.float64, device=torch.cuda.current_device())
    else:
        t = torch.tensor([(time.perf_counter() - state["t0"]) * 1e3], dtype=torch.float64)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def stage_plan(runner: ModelRunner, plan) -> Tuple[object, int, int]:
    """Worker side: copy a received plan into the runner's staging buffers."""
    from rusteeze_b200.engine.model_runner import choose_num_splits
    from rusteeze_b200.models.decoder import AttentionMetadata
    r = runner
    T, S, MB = plan["T"], plan["S"], plan["mb"]
    # alternate the pinned staging sets as rank 0 does: with pipelined steps this plan
    # arrives while the previous step's host->device copies (and its sample-row index
    # copy) may still be queued on the stream, reading the other set
    r._flip_host()
    r.h_input_ids[:T] = torch.from_numpy(plan["ids"])
    r.h_positions[:T] = torch.from_numpy(plan["pos"])
    r.h_slots[:T] = torch.from_numpy(plan["slots"])
    r.h_qsl[:S + 1] = torch.from_numpy(plan["qsl"])
    r.h_seq_lens[:S] = torch.from_numpy(plan["sl"])
    r.h_block_tables[:S].zero_()
    r.h_block_tables[:S, :MB] = torch.from_numpy(plan["bt"])
    nb = r.is_cuda
    r.d_input_ids[:T].copy_(r.h_input_ids[:T], non_blocking=nb)
    r.d_positions[:T].copy_(r.h_positions[:T], non_blocking=nb)
    r.d_slots[:T].copy_(r.h_slots[:T], non_blocking=nb)
    r.d_qsl[:S + 1].copy_(r.h_qsl[:S + 1], non_blocking=nb)
    r.d_seq_lens[:S].copy_(r.h_seq_lens[:S], non_blocking=nb)
    r.d_block_tables[:S].copy_(r.h_block_tables[:S], non_blocking=nb)
    meta = AttentionMetadata(
        num_seqs=S, num_tokens=T, num_decode_seqs=plan["nd"], query_start_loc=r.d_qsl[:S + 1],
        seq_lens=r.d_seq_lens[:S], block_tables=r.d_block_tables[:S], slot_mapping=r.d_slots[:T],
        max_query_len=plan["maxq"], max_seq_len=plan["maxs"],
        decode_num_splits=choose_num_splits(max(plan["nd"], 1), r.model.hkv, r.max_blocks),
        decode_workspace=r.decode_ws, prefill_kv_blocks=r.prefill_kv_blocks(plan["nd"], S))
    if not r.is_cuda:
        meta.query_start_loc = r.h_qsl[:S + 1].clone()
        meta.seq_lens = r.h_seq_lens[:S].clone()
        meta.block_tables = r.h_block_tables[:S].clone()
    return meta, T, S


@torch.no_grad()
def worker_loop(runner: ModelRunner, channel: PlanChannel, idle_timeout_s: float = 600.0) -> int:
    """Runs plans until rank 0 sends STOP or closes the ring.  Returns steps run."""
    steps = 0
    timer_state: dict = {}
    idle_since = time.monotonic()
    while True:
        msg = channel.consume(1.0)
        if msg is None:
            if channel.ring.closed:
                return steps
            if time.monotonic() - idle_since > idle_timeout_s:
                log.error("worker %d: no plan from rank 0 for %.0f s, exiting", channel.rank, idle_timeout_s)
                return steps
            continue
        idle_since = time.monotonic()
        kind, plan = msg
        if kind == MSG_STOP:
            return steps
        if "capture" in plan:
            runner.capture_graphs(plan["capture"])
            continue
        if "timer" in plan:
            _timer_mark(runner, plan["timer"], timer_state)
            continue
        if "blockops" in plan:
            sout, sin, copy = plan["blockops"]
            if sout:
                runner.swap_out(sout)
            if sin:
                runner.swap_in(sin)
            if copy:
                runner.copy_blocks(copy)
            continue
        if "arrays" in plan:
            meta, T, S = stage_plan(runner, plan)
            n_rows = plan["arrays"]
            runner.h_logits_idx[:n_rows] = torch.from_numpy(plan["lidx"][:n_rows])
            runner.forward_staged(meta, T, n_rows)
            steps += 1
            continue
        if plan["sout"]:
            runner.swap_out(plan["sout"])
        if plan["sin"]:
            runner.swap_in(plan["sin"])
        if plan["copy"]:
            runner.copy_blocks(plan["copy"])
        prev = None
        if plan.get("bcast"):
            # pipelined steps: rank 0's previous sample tensor, for the decode inputs below
            import torch.distributed as dist
            prev = torch.empty(plan["bcast"], dtype=torch.int64, device=runner.device)
            dist.broadcast(prev, src=0)
        meta, T, S = stage_plan(runner, plan)
        if prev is not None:
            dst, src = plan["pend"]
            idx = torch.tensor(dst + src, dtype=torch.int64).to(runner.device, non_blocking=runner.is_cuda)
            runner.d_input_ids.index_copy_(0, idx[:len(dst)], prev.index_select(0, idx[len(dst):]))
        runner.forward_logits(meta, T, S, plan["rows"], pure_decode=plan["pure"])
        steps += 1
