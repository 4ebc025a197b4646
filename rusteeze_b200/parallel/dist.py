"""Process groups and the tensor-parallel communicator.

One process per GPU (torchrun-style env: RANK, WORLD_SIZE, LOCAL_RANK,
MASTER_ADDR, MASTER_PORT).  The reference declares `TensorParallelConfig`
with an in-process backend and an NCCL backend marked "future", and its
collectives are no-ops (crates/rusteeze-engine/src/tensor_parallel.rs:28-106).
Here `TPComm` is the real thing:

  * mode "nccl":  torch.distributed collectives (NCCL on GPUs, gloo on CPU
                  ranks for tests) -- the baseline.
  * mode "fused": the peer-memory kernels: one-shot / two-shot all-reduce
                  over NVLink P2P (`parallel.comm`) and, for dense models,
                  layer boundaries fused with their collectives
                  (`parallel.fused_tp`: GEMM epilogues that reduce-scatter
                  straight into the owners' buffers, add+RMSNorm+all-gather,
                  GEMMs that start on gathered tiles as they land).

Every process group is created with a short timeout so that a dead rank
turns into an error on the survivors instead of a hang.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta
from typing import Optional

import torch
import torch.distributed as dist

from rusteeze_b200 import ops
from rusteeze_b200.models.decoder import TPGroup


@dataclass
class DistInfo:
    rank: int
    world_size: int
    local_rank: int
    device: torch.device
    backend: str


def init_distributed(backend: Optional[str] = None, timeout_s: float = 120.0,
                     device_type: Optional[str] = None) -> DistInfo:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    dt = device_type or ("cuda" if torch.cuda.is_available() else "cpu")
    backend = backend or ("nccl" if dt == "cuda" else "gloo")
    device = torch.device(dt, local) if dt == "cuda" else torch.device("cpu")
    if dt == "cuda":
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        kw = dict(backend=backend, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(**kw)
    return DistInfo(rank, world, local, device, backend)


class TPComm(TPGroup):
    """Tensor-parallel communicator handed to the model."""

    def __init__(self, rank: int, size: int, group=None, mode: str = "nccl", device=None,
                 max_tokens: int = 8192, hidden: int = 4096):
        self.rank, self.size = rank, size
        self.group = group
        self.mode = mode
        self.device = device
        self.fused = None
        self.fused_tp = None
        if mode == "fused" and size > 1 and device is not None and torch.device(device).type == "cuda":
            from rusteeze_b200.parallel.comm import PeerAllReduce
            from rusteeze_b200.parallel.fused_tp import FusedTP
            self.fused = PeerAllReduce(group, rank, size, torch.device(device), max_tokens * hidden)
            if hidden % 256 == 0:
                # layer boundaries: GEMM + reduce-scatter -> add + RMSNorm + all-gather -> GEMM
                self.fused_tp = FusedTP(group, rank, size, torch.device(device), max_tokens, hidden)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        if self.fused is not None and x.is_cuda and self.fused.fits(x):
            return self.fused.all_reduce(x)
        dist.all_reduce(x, group=self.group)
        return x

    def all_gather_last_dim(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        n, v = x.shape
        if x.is_cuda:
            out = torch.empty(self.size, n, v, dtype=x.dtype, device=x.device)
            dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
            return out.permute(1, 0, 2).reshape(n, self.size * v)
        parts = [torch.empty_like(x) for _ in range(self.size)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

    def row_parallel_linear(self, x, w, bias=None):
        if self.fused is not None and x.is_cuda and x.shape[0] > 0:
            return self.fused.linear_all_reduce(x, w, bias)
        y = ops.linear(x, w, bias if self.rank == 0 else None)
        return self.all_reduce(y)

    def barrier(self) -> None:
        if self.size > 1:
            dist.barrier(group=self.group)
