"""Peer-memory collectives for tensor parallelism (NVLink P2P over NVSwitch).

`PeerAllReduce` allocates one symmetric buffer per rank with torch
symmetric memory (every rank maps every peer's buffer), and runs the
sm_100a `peer_all_reduce` kernel (csrc/kernels/comm.cu): one-shot for
small (decode-sized) messages, two-shot reduce-scatter + all-gather for
larger ones, per-block epoch flags with bounded acquire spins.  No library
kernel ever touches a peer pointer; NCCL stays the baseline
(`comm_backend: nccl`).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from rusteeze_b200 import ops

TWO_SHOT_BYTES = 256 * 1024


class PeerAllReduce:
    def __init__(self, group, rank: int, world: int, device: torch.device, max_elems: int):
        import torch.distributed._symmetric_memory as symm
        C = ops.cuda_ext()
        self.rank, self.world, self.device = rank, world, device
        self.group = group or dist.group.WORLD
        flag = int(C.peer_flag_bytes())
        self.half = ((max_elems * 2 + 255) // 256) * 256
        try:
            symm.enable_symm_mem_for_group(self.group.group_name)
        except Exception:  # noqa: BLE001 -- newer torch enables it implicitly
            pass
        self.buf = symm.empty(flag + 2 * self.half, dtype=torch.uint8, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.handle = symm.rendezvous(self.buf, self.group)
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        dist.barrier(group=self.group)

    def fits(self, x: torch.Tensor) -> bool:
        n = x.numel()
        return x.dtype == torch.bfloat16 and n % (8 * self.world) == 0 and n * 2 <= self.half

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        x = x.contiguous()
        out = torch.empty_like(x)
        two = x.numel() * 2 >= TWO_SHOT_BYTES
        ops.add_launches(ops.cuda_ext().peer_all_reduce(out, x, self.ptrs, self.rank, self.half, self.epoch,
                                                        self.status, two))
        return out

    def linear_all_reduce(self, x: torch.Tensor, w: torch.Tensor, bias=None) -> torch.Tensor:
        y = ops.linear(x, w, bias if self.rank == 0 else None)
        if self.fits(y):
            return self.all_reduce(y)
        dist.all_reduce(y, group=self.group)
        return y

    def check(self) -> int:
        return int(self.status[0])
