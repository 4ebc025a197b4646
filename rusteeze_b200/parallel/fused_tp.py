"""Tensor-parallel layer boundaries fused with their collectives.

Megatron-style TP normally ends every row-parallel GEMM (o_proj, down_proj)
with an all-reduce and then runs residual-add + RMSNorm on every rank.  Here
the residual stream between layers is sequence-sharded (rank o owns rows
[o*R, (o+1)*R), R = rs_rows) and the collective is folded into the kernels
around it (csrc/kernels/tp_fused.cu, gemm_bf16.cu):

  gemm_rs      row-parallel GEMM; its epilogue stores every finished tile row
               into the owner's slot buffer over NVLink (reduce-scatter);
  rs_norm_ag   the owner sums its slots in fp32, adds its residual shard,
               RMS-normalises and stores the rows into every rank's gather
               buffer (all-gather);
  gemm_ag      the next column-parallel GEMM reads the gathered rows from
               LOCAL memory; its TMA producer waits per A tile for the rows'
               all-gather flags, so it starts as soon as its rows landed;
  moe          expert parallelism (Mixtral): the all-gather above is the
               dispatch (every rank sees every token); each rank runs its own
               experts and its combine kernel stores every weighted expert
               output row straight into the owner's slot k over NVLink, so the
               owner's rs_norm_ag sums top-k slots instead of world partials.
  MXFP8        with block-scaled FP8 weights the same chain runs on the
               block-scaled GEMMs: rs_norm_ag quantises the normalised rows
               (e4m3 + power-of-two 1x128 scales in the GEMM's scale-chunk
               layout) before the all-gather, which halves its NVLink bytes,
               and the gate/up GEMM's SiLU epilogue emits the down projection's
               operand (gemm_rs_mx / gemm_ag_mx).

One symmetric allocation per rank (torch symmetric memory) holds
[rs flags | ag flags | moe flags | slots | gather | gather e4m3 | gather
scales]; peers' bases come from the rendezvous.  The reference has no collective at all
(crates/rusteeze-engine/src/tensor_parallel.rs:80-106).
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from rusteeze_b200 import ops

_ALIGN = 1024


def _up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class FusedTP:
    def __init__(self, group, rank: int, world: int, device: torch.device, max_tokens: int, hidden: int):
        import torch.distributed._symmetric_memory as symm
        self.group = group or dist.group.WORLD
        self.rank, self.world, self.device, self.hidden = rank, world, device, hidden
        self.max_tokens = max_tokens
        self.max_rs_rows = _up(-(-max_tokens // world), 8)
        self.max_m_tiles = -(-max_tokens // 128) + 1
        self.max_n_tiles = -(-hidden // 64)          # n tiles of a row-parallel output at the smallest tile
        n_rs_flags = self.max_m_tiles * self.max_n_tiles * 8 * world   # [m tile][n tile][quarter x half][src]
        n_ag_flags = -(-max_tokens // 8) + 16
        n_moe_flags = 8 * self.max_rs_rows                 # [topk <= 8][rs_rows]
        self.off_rs_flag = 0
        self.off_ag_flag = _up(self.off_rs_flag + 4 * n_rs_flags, _ALIGN)
        self.off_moe_flag = _up(self.off_ag_flag + 4 * n_ag_flags, _ALIGN)
        self.off_slots = _up(self.off_moe_flag + 4 * n_moe_flags, _ALIGN)
        self.off_gather = _up(self.off_slots + 2 * world * self.max_rs_rows * hidden, _ALIGN)
        # MXFP8 all-gather: e4m3 rows and their UE8M0 scale chunks (block-scaled GEMM layout)
        self.mx_ok = hidden % 128 == 0
        self.n_sf_bytes = (self.max_m_tiles + 1) * (hidden // 128) * 512 if self.mx_ok else 0
        self.off_gather_q = _up(self.off_gather + 2 * (max_tokens + 128) * hidden, _ALIGN)
        self.off_gather_sf = _up(self.off_gather_q + ((max_tokens + 128) * hidden if self.mx_ok else 0), _ALIGN)
        total = _up(self.off_gather_sf + self.n_sf_bytes, _ALIGN)
        try:
            symm.enable_symm_mem_for_group(self.group.group_name)
        except Exception:  # noqa: BLE001 -- newer torch enables it implicitly
            pass
        self.buf = symm.empty(total, dtype=torch.uint8, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.handle = symm.rendezvous(self.buf, self.group)
        bases = [int(p) for p in self.handle.buffer_ptrs]
        self.slot_ptrs = [b + self.off_slots for b in bases]
        self.rs_flag_ptrs = [b + self.off_rs_flag for b in bases]
        self.gather_ptrs = [b + self.off_gather for b in bases]
        self.ag_flag_ptrs = [b + self.off_ag_flag for b in bases]
        self.moe_flag_ptrs = [b + self.off_moe_flag for b in bases]
        self.gather_q_ptrs = [b + self.off_gather_q for b in bases] if self.mx_ok else []
        self.gather_sf_ptrs = [b + self.off_gather_sf for b in bases] if self.mx_ok else []
        u8 = self.buf
        self.rs_flag = u8[self.off_rs_flag:self.off_rs_flag + 4 * n_rs_flags].view(torch.int32)
        self.ag_flag = u8[self.off_ag_flag:self.off_ag_flag + 4 * n_ag_flags].view(torch.int32)
        self.moe_flag = u8[self.off_moe_flag:self.off_moe_flag + 4 * n_moe_flags].view(torch.int32)
        self.slots = u8[self.off_slots:self.off_slots + 2 * world * self.max_rs_rows * hidden].view(torch.bfloat16)
        self.gather = u8[self.off_gather:self.off_gather + 2 * (max_tokens + 128) * hidden].view(
            torch.bfloat16).view(max_tokens + 128, hidden)
        if self.mx_ok:
            self.gather_q = u8[self.off_gather_q:self.off_gather_q + (max_tokens + 128) * hidden].view(
                torch.float8_e4m3fn).view(max_tokens + 128, hidden)
            self.gather_sf = u8[self.off_gather_sf:self.off_gather_sf + self.n_sf_bytes]
        self.residual = torch.empty(self.max_rs_rows, hidden, dtype=torch.bfloat16, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.n_tiles = 1
        # race testing of the flag protocols: RZ_TP_JITTER_NS=<ns> makes the communication
        # kernels pause pseudo-randomly before their peer stores and flag releases
        jitter = int(os.environ.get("RZ_TP_JITTER_NS", "0") or 0)
        if jitter:
            ops.cuda_ext().set_comm_jitter_ns(jitter)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ shapes
    def rs_rows(self, M: int) -> int:
        return _up(-(-M // self.world), 8)

    def fits(self, M: int) -> bool:
        # the add+RMSNorm+all-gather kernel keeps a row in registers: hidden <= 8192, 8-column chunks
        return 0 < M <= self.max_tokens and self.hidden <= 8192 and self.hidden % 8 == 0

    # ------------------------------------------------------------------ ops
    def _mx_args(self, mx: bool):
        if mx and not self.mx_ok:
            raise ValueError("MXFP8 all-gather needs hidden % 128 == 0")
        return (self.gather_q_ptrs, self.gather_sf_ptrs) if mx else ([], [])

    def _gathered(self, M: int, mx: bool):
        return (self.gather_q[:M], self.gather_sf) if mx else self.gather[:M]

    def start(self, h: torch.Tensor, norm_w: torch.Tensor, eps: float, offset: float, mx: bool = False):
        """First boundary: x = h (replicated rows), residual shard = own rows,
        normalised rows all-gathered.  Returns the gathered [M, H] view, or with
        `mx` the MXFP8 operand (e4m3 [M, H] view, scale chunks)."""
        M = h.shape[0]
        C = ops.cuda_ext()
        gq, gsf = self._mx_args(mx)
        C.rs_norm_ag(self.slots, self.rs_flag, 1, h.contiguous(), self.residual, norm_w, eps, offset,
                     self.gather_ptrs, self.ag_flag_ptrs, self.rank, M, self.rs_rows(M), self.epoch, 0, 0, None,
                     gq, gsf)
        ops.add_launches(1)
        return self._gathered(M, mx)

    def moe(self, g: torch.Tensor, router: torch.Tensor, w13_il: torch.Tensor, w2: torch.Tensor, topk: int,
            e_lo: int, call_idx_in: int, call_idx: int) -> None:
        """Expert-parallel MoE on the all-gathered rows: waits for the rows of
        boundary `call_idx_in`, runs this rank's experts, and sends every
        weighted expert output row to its token's owner (slot k) with a flag;
        `rs_norm_ag(..., moe_topk=topk)` then sums the slots on the owner."""
        M = g.shape[0]
        C = ops.cuda_ext()
        C.ag_wait(self.ag_flag, M, self.epoch, call_idx_in)
        ops.add_launches(1)
        ops.add_launches(C.moe_forward_peer(g, router, w13_il, w2, topk, e_lo, True, self.slot_ptrs,
                                            self.moe_flag_ptrs, self.rs_rows(M), self.epoch, call_idx))

    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor, call_idx: int) -> None:
        M = x.shape[0]
        self.n_tiles = int(ops.cuda_ext().gemm_peer_rs(x.contiguous(), w, self.slot_ptrs, self.rs_flag_ptrs,
                                                       self.rank, self.rs_rows(M), self.epoch, call_idx, 0))
        ops.add_launches(1)

    def rs_norm_ag(self, M: int, norm_w: torch.Tensor, eps: float, offset: float, call_idx: int,
                   moe_topk: int = 0, mx: bool = False):
        gq, gsf = self._mx_args(mx)
        ops.cuda_ext().rs_norm_ag(self.slots, self.rs_flag, self.n_tiles, None, self.residual, norm_w, eps, offset,
                                  self.gather_ptrs, self.ag_flag_ptrs, self.rank, M, self.rs_rows(M), self.epoch,
                                  call_idx, moe_topk, self.moe_flag if moe_topk else None, gq, gsf)
        ops.add_launches(1)
        return self._gathered(M, mx)

    def gemm_rs_mx(self, xq: torch.Tensor, sfa: torch.Tensor, wq: torch.Tensor, wsf: torch.Tensor,
                   call_idx: int) -> None:
        """MXFP8 row-parallel GEMM (operand from `ops.quant_mxf8_act` or a SiLU-quantising
        epilogue) reduce-scattering its bf16 rows into the owners' slots."""
        M = xq.shape[0]
        self.n_tiles = int(ops.cuda_ext().gemm_peer_rs_mx(xq, sfa, wq, wsf, self.slot_ptrs, self.rs_flag_ptrs,
                                                          self.rank, self.rs_rows(M), self.epoch, call_idx))
        ops.add_launches(1)

    def gemm_ag_mx(self, g, wq: torch.Tensor, wsf: torch.Tensor, call_idx: int,
                   bias: Optional[torch.Tensor] = None, silu_q: bool = False):
        """MXFP8 GEMM on the all-gathered operand `g` = (e4m3 rows, scale chunks):
        bf16 [M, N] rows, or with `silu_q` (gate/up, rows interleaved in 64-row
        blocks) SiLU(gate)*up as the next MXFP8 operand (e4m3 [M, N/2], scales)."""
        gq, gsf = g
        M, N = gq.shape[0], wq.shape[0]
        if silu_q:
            q = torch.empty(M, N // 2, dtype=torch.float8_e4m3fn, device=gq.device)
            sf = torch.empty((M + 127) // 128, N // 256, 512, dtype=torch.uint8, device=gq.device)
            ops.add_launches(ops.cuda_ext().gemm_mxf8_ag(q, sf, gq, gsf, wq, wsf, bias, self.ag_flag, self.epoch,
                                                         call_idx))
            return q, sf
        out = torch.empty(M, N, dtype=torch.bfloat16, device=gq.device)
        ops.add_launches(ops.cuda_ext().gemm_mxf8_ag(out, None, gq, gsf, wq, wsf, bias, self.ag_flag, self.epoch,
                                                     call_idx))
        return out

    def gemm_ag(self, g: torch.Tensor, w: torch.Tensor, call_idx: int, bias: Optional[torch.Tensor] = None,
                silu_mul: bool = False, act: str = "silu") -> torch.Tensor:
        """GEMM on the gathered rows; with silu_mul the gated epilogue applies `act`
        (SiLU, or GELU-tanh for GeGLU MLPs) to interleaved gate/up weight rows."""
        M = g.shape[0]
        n_out = w.shape[0] // 2 if silu_mul else w.shape[0]
        out = torch.empty(M, n_out, dtype=torch.bfloat16, device=g.device)
        epi = (1 | ops._gate(act)) if silu_mul else 0
        ops.add_launches(ops.cuda_ext().gemm_ag(out, g, w, bias, epi, self.ag_flag, self.epoch, call_idx))
        return out

    def wait_gathered(self, M: int, call_idx: int) -> None:
        """Waits (bounded, on the device) until every owner's rows of boundary `call_idx`
        have landed in the local gather buffer; a consumer that is not a flag-waiting
        GEMM (the LM head reads the final boundary's rows) needs it."""
        ops.cuda_ext().ag_wait(self.ag_flag, M, self.epoch, call_idx)
        ops.add_launches(1)

    def end_step(self) -> None:
        ops.cuda_ext().tp_epoch_bump(self.epoch)
        ops.add_launches(1)
