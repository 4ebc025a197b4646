"""Bring-up of a tensor-parallel engine: one process per GPU.

`tp_rank_setup` is what every rank runs (under torchrun or the spawner
below): init the process group, build this rank's weight shard, agree on
the KV block count (MIN over ranks of what each GPU can hold), build the
ModelRunner and the plan channel.  Rank 0 then wraps its runner in a
`TPExecutor` and builds the `LLMEngine`; other ranks enter `worker_loop`.

`TPEngineLauncher` spawns ranks 1..N-1 from the serving process (used by
`rusteeze serve --tensor-parallel-size N`).
"""
from __future__ import annotations

import copy
import logging
import os
import socket
from typing import Optional

import torch
import torch.distributed as dist

from rusteeze_b200.config.config import Config
from rusteeze_b200.engine.model_runner import ModelRunner
from rusteeze_b200.models.config import ModelConfig, get_preset
from rusteeze_b200.models.loader import build_model
from rusteeze_b200.parallel.dist import DistInfo, TPComm, init_distributed
from rusteeze_b200.parallel.executor import PlanChannel, TPExecutor, worker_loop

log = logging.getLogger("rusteeze.tp")


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model_config(cfg: Config) -> ModelConfig:
    mc = cfg.model
    return ModelConfig.from_json_file(mc.path) if mc.path else get_preset(mc.preset or "tiny-llama")


def tp_rank_setup(cfg: Config, info: DistInfo, model_config: Optional[ModelConfig] = None, tag: str = "0",
                  liveness=None, build_engine: bool = True):
    """Builds this rank's shard, runner and plan channel.  Rank 0 returns (engine, runner,
    channel); with build_engine=False (worker-group recovery) it returns (executor, runner,
    channel) for an engine that already exists."""
    from rusteeze_b200.engine.llm_engine import LLMEngine, _dtype, kv_cache_dtype
    mc = model_config or _model_config(cfg)
    ec = cfg.engine
    dev = str(info.device)
    dtype = _dtype(cfg.model.dtype, dev)
    kv_dtype = kv_cache_dtype(ec.kv_cache_dtype, dtype)
    max_len = min(cfg.model.max_model_len or mc.max_position_embeddings, mc.max_position_embeddings)
    tp = TPComm(info.rank, info.world_size, group=dist.group.WORLD if info.world_size > 1 else None,
                mode=ec.comm_backend if info.device.type == "cuda" else "nccl", device=info.device,
                max_tokens=max(ec.max_num_batched_tokens, ec.max_num_seqs), hidden=mc.hidden_size)
    # MoE: attention is tensor-parallel, the experts are split over the same ranks (expert
    # parallelism); every rank routes all tokens and the partial outputs are summed
    ep_rank, ep_size = (info.rank, info.world_size) if mc.is_moe else (0, 1)
    model = build_model(mc, dtype=dtype, device=dev, tp=tp, ep_rank=ep_rank, ep_size=ep_size,
                        model_dir=cfg.model.path, seed=cfg.model.seed)
    q = cfg.model.quantization
    if q is not None and q.method != "none":
        # block-scaled FP8 of this rank's shard (every sharded K / N is a multiple of 128)
        from rusteeze_b200.models.quant import quantize_model_fp8
        quantize_model_fp8(model, getattr(q, "scale_format", "ue8m0"))
    if info.device.type == "cuda":
        model.prepare_for_gpu()
    # agree on the KV block count
    if ec.num_gpu_blocks:
        nblocks = ec.num_gpu_blocks
    elif info.device.type == "cuda":
        free, total = torch.cuda.mem_get_info()
        budget = total * ec.gpu_memory_utilization - (total - free) - 4 * (1 << 30)
        per_block = 2 * mc.num_hidden_layers * model.hkv * mc.head_dim * 16 * torch.finfo(kv_dtype).bits // 8
        if info.rank == 0:
            # rank 0 also holds the unsharded draft model of speculative decoding and its KV
            from rusteeze_b200.engine.spec_decode import draft_memory
            d_w, d_blk = draft_memory(mc, ec.speculative, torch.finfo(dtype).bits // 8, 16)
            budget -= d_w
            per_block += d_blk
        nblocks = int(budget // per_block)
    else:
        nblocks = 256
    if info.world_size > 1:
        t = torch.tensor([nblocks], dtype=torch.int64, device=info.device if info.backend == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        nblocks = int(t.item())
    from rusteeze_b200.engine.llm_engine import swap_blocks
    n_swap = swap_blocks(ec, mc, kv_dtype, dev)     # the same count on every rank and in rank 0's engine
    runner = ModelRunner(model, num_gpu_blocks=nblocks, num_cpu_blocks=n_swap, max_num_seqs=ec.max_num_seqs,
                         max_num_batched_tokens=ec.max_num_batched_tokens, max_model_len=max_len,
                         kv_dtype=kv_dtype, use_cuda_graph=not ec.enforce_eager, seed=cfg.model.seed)
    channel = None
    if info.world_size > 1:
        if info.rank == 0:
            channel = PlanChannel(tag, 0, info.world_size)
        dist.barrier()
        if info.rank != 0:
            channel = PlanChannel(tag, info.rank, info.world_size)
        dist.barrier()
    ecfg = copy.deepcopy(cfg)
    ecfg.engine.num_gpu_blocks = nblocks
    ecfg.model.device = dev
    if info.rank == 0:
        executor = TPExecutor(runner, channel, liveness) if channel is not None else runner
        if not build_engine:
            return executor, runner, channel
        engine = LLMEngine(ecfg, model=model, executor=executor)
        return engine, runner, channel
    return None, runner, channel


def tp_worker_main(cfg: Config, info: DistInfo, model_config: Optional[ModelConfig] = None, tag: str = "0") -> int:
    _, runner, channel = tp_rank_setup(cfg, info, model_config, tag)
    try:
        steps = worker_loop(runner, channel)
    finally:
        runner.release_graphs()        # graphs holding NCCL calls block destroy_process_group
    return steps


def _spawned_worker(rank: int, world: int, port: int, cfg_dict: dict, mc_dict: Optional[dict], tag: str,
                    device_type: str) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    wd = float(os.environ.get("RZ_WORKER_WATCHDOG_S", "0") or 0)
    if wd > 0:
        # diagnostics: a worker stuck for `wd` seconds prints every thread's stack and exits
        import faulthandler
        faulthandler.dump_traceback_later(wd, exit=True)
    from rusteeze_b200.config.config import config_from_dict
    cfg = config_from_dict(cfg_dict)
    mc = ModelConfig(**mc_dict) if mc_dict else None
    info = init_distributed(device_type=device_type, timeout_s=float(os.environ.get("RZ_PG_TIMEOUT_S", "120")))
    try:
        tp_worker_main(cfg, info, mc, tag)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


class TPEngineLauncher:
    """Spawns ranks 1..N-1 and builds rank 0's engine in this process.

    Worker-group recovery: when a worker process dies (the engine's next step raises
    DistributedError before it publishes a plan), `recover()` tears the group down,
    spawns a fresh set of workers on a new rendezvous, rebuilds rank 0's shard, runner and
    plan channel, and hands them to the existing engine, which re-queues every live
    sequence as a recompute preemption (the KV cache went with the old group).  Requests
    in flight then complete as if they had been preempted.  The reference handles
    failures only by request timeout, abort and shutdown
    (crates/rusteeze-engine/src/engine.rs:295,575-603)."""

    def __init__(self, cfg: Config, model_config: Optional[ModelConfig] = None, device_type: Optional[str] = None):
        self.cfg = cfg
        self.model_config = model_config
        self.world = cfg.model.tensor_parallel_size
        self.device_type = device_type or ("cuda" if torch.cuda.is_available() else "cpu")
        self.recoveries = 0
        info = self._spawn()
        self._engine, self.runner, self.channel = tp_rank_setup(cfg, info, model_config, self.tag,
                                                                liveness=self.dead_workers)
        self._engine.tp_launcher = self

    def _spawn(self) -> DistInfo:
        import torch.multiprocessing as mp
        port = free_port()
        self.tag = f"{os.getpid()}_{port}"
        ctx = mp.get_context("spawn")
        mc_dict = self.model_config.to_dict() if self.model_config else None
        self.procs = [ctx.Process(target=_spawned_worker, args=(r, self.world, port, self.cfg.to_dict(), mc_dict,
                                                                 self.tag, self.device_type), daemon=True)
                      for r in range(1, self.world)]
        for p in self.procs:
            p.start()
        # the rendezvous variables are set for the process group's creation only: left in
        # this process's environment they would make every later child (a tool, a test's
        # subprocess) believe it is rank 0 of this group
        env = dict(RANK="0", WORLD_SIZE=str(self.world), LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port))
        saved = {k: os.environ.get(k) for k in env}
        os.environ.update(env)
        try:
            return init_distributed(device_type=self.device_type,
                                    timeout_s=float(os.environ.get("RZ_PG_TIMEOUT_S", "120")))
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v

    def dead_workers(self):
        """Ranks whose worker process has exited."""
        return [r for r, p in enumerate(self.procs, start=1) if not p.is_alive()]

    def engine(self):
        return self._engine

    def _teardown(self, timeout: float) -> None:
        for p in self.procs:
            p.join(timeout)
            if p.is_alive():
                p.terminate()
                p.join(timeout)
        if self.channel is not None:
            try:
                self.channel.close()
            except Exception:  # noqa: BLE001 -- already closed
                pass
        # graphs holding collectives must go before the process group, on every rank
        self.runner.release_graphs()
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception as e:  # noqa: BLE001 -- a group with a dead member may not close cleanly
                log.warning("process group teardown after a worker failure: %r", e)

    def recover(self) -> None:
        """Replaces the worker group after a worker died (see the class docstring)."""
        dead = self.dead_workers()
        log.error("tensor-parallel worker rank(s) %s died; restarting the worker group", dead)
        try:
            self.channel.ring.close()          # surviving workers see the closed ring and exit
        except Exception:  # noqa: BLE001
            pass
        self._teardown(timeout=10.0)
        info = self._spawn()
        executor, self.runner, self.channel = tp_rank_setup(self.cfg, info, self.model_config, self.tag,
                                                            liveness=self.dead_workers, build_engine=False)
        self._engine.recover_from_worker_failure(executor, self.runner.num_gpu_blocks)
        self.recoveries += 1

    def shutdown(self, timeout: float = 30.0) -> None:
        if self.channel is not None:
            try:
                self._engine.runner.shutdown()
            except Exception:  # noqa: BLE001 -- a dead worker cannot consume the stop message
                pass
        self.runner.release_graphs()
        for p in self.procs:
            p.join(timeout)
            if p.is_alive():
                p.terminate()
        if dist.is_initialized():
            dist.destroy_process_group()
