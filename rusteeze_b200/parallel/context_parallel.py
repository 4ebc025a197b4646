"""Context-parallel (ring) attention for long-prompt prefill.

One sequence's tokens are split over the ranks of a process group; every rank keeps the
queries, keys and values of its own tokens.  The key/value chunks travel around the ring
(world - 1 point-to-point exchanges, each overlapped with the attention of the chunk in
hand), every rank attends its queries to each chunk it sees, and the partial results are
merged with their log-sum-exp.  Causal masking uses absolute token positions, so any split
works; `zigzag_split` gives rank r the chunks r and 2 world - 1 - r of 2 world equal pieces,
which balances the causal work (early chunks see few keys, late ones many).

This is a library operation (a stretch item of the component list: the reference has no
context parallelism).  The serving engine shards heads (tensor parallelism), not tokens,
and does not call it; the math runs in fp32 torch on whatever device the tensors are on.
Tested on gloo ranks against the dense oracle (tests/test_context_parallel.py).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def zigzag_split(num_tokens: int, world: int) -> List[List[Tuple[int, int]]]:
    """Per rank, the token ranges [start, end) it owns: the sequence cut into 2 * world
    near-equal pieces, rank r taking pieces r and 2 * world - 1 - r."""
    n = 2 * world
    bounds = [round(i * num_tokens / n) for i in range(n + 1)]
    return [[(bounds[r], bounds[r + 1]), (bounds[n - 1 - r], bounds[n - r])] for r in range(world)]


def positions_of(ranges: List[Tuple[int, int]]) -> torch.Tensor:
    return torch.cat([torch.arange(a, b) for a, b in ranges]) if ranges else torch.zeros(0, dtype=torch.long)


def attention_partial(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor,
                      k_pos: torch.Tensor, scale: float, causal: bool = True, window: Optional[int] = None,
                      softcap: Optional[float] = None, alibi: Optional[torch.Tensor] = None):
    """Normalised attention output o [Tq, Hq, D] of q over this key chunk, and the
    log-sum-exp lse [Tq, Hq] of its logits (-inf where a query sees no key of the chunk).
    Keys with Hkv < Hq heads are shared by groups of Hq / Hkv query heads (GQA)."""
    hq, hkv = q.shape[1], k.shape[1]
    g = hq // hkv
    K = k.float().repeat_interleave(g, dim=1)
    V = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), K) * scale
    if softcap:
        s = softcap * torch.tanh(s / softcap)
    qp = q_pos.view(-1, 1).to(s.device)
    kp = k_pos.view(1, -1).to(s.device)
    if alibi is not None:
        s = s + alibi.float().to(s.device).view(-1, 1, 1) * (kp - qp).float().unsqueeze(0)
    mask = torch.zeros(qp.shape[0], kp.shape[1], dtype=torch.bool, device=s.device)
    if causal:
        mask |= kp > qp
    if window:
        mask |= kp <= qp - window
    s = s.masked_fill(mask.unsqueeze(0), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)                                       # [H, Tq]
    p = torch.exp(s - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse).unsqueeze(-1))
    o = torch.einsum("hqk,khd->qhd", p, V)
    return o, lse.t().contiguous()


def merge_partials(o1: torch.Tensor, lse1: torch.Tensor, o2: torch.Tensor, lse2: torch.Tensor):
    """Combines two normalised partial attentions over disjoint key sets:
    o = (e^lse1 o1 + e^lse2 o2) / (e^lse1 + e^lse2), lse = log(e^lse1 + e^lse2)."""
    m = torch.maximum(lse1, lse2)
    m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w1, w2 = torch.exp(lse1 - m), torch.exp(lse2 - m)
    den = w1 + w2
    safe = torch.where(den > 0, den, torch.ones_like(den))
    o = (o1 * w1.unsqueeze(-1) + o2 * w2.unsqueeze(-1)) / safe.unsqueeze(-1)
    lse = torch.where(den > 0, m + torch.log(safe), torch.full_like(den, float("-inf")))
    return o, lse


def _exchange(tensors: List[torch.Tensor], bufs: List[torch.Tensor], nxt: int, prv: int, nccl: bool):
    """Starts sending `tensors` to rank `nxt` and receiving `bufs` from rank `prv`; returns
    the request handles."""
    if nccl:
        ops = [dist.P2POp(dist.isend, t, nxt) for t in tensors] + [dist.P2POp(dist.irecv, b, prv) for b in bufs]
        return dist.batch_isend_irecv(ops)
    return [dist.isend(t, nxt) for t in tensors] + [dist.irecv(b, prv) for b in bufs]


@torch.no_grad()
def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, k_pos: torch.Tensor,
                   scale: float, group=None, causal: bool = True, window: Optional[int] = None,
                   softcap: Optional[float] = None, alibi: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of this rank's queries q [Tq, Hq, D] (absolute positions q_pos) over the
    keys / values of every rank of `group` (this rank's k, v [Tk, Hkv, D] at k_pos).  The
    key chunks circulate around the ring; each step sends the chunk in hand onwards while
    attending to it.  Chunks wholly in the future of every local query are passed on
    without being attended.  Returns o [Tq, Hq, D] in q's dtype."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    o, lse = attention_partial(q, k, v, q_pos, k_pos, scale, causal, window, softcap, alibi)
    if world == 1:
        return o.to(q.dtype)
    rank = dist.get_rank(group)
    gr = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    nxt, prv = gr((rank + 1) % world), gr((rank - 1) % world)
    nccl = dist.get_backend(group) == "nccl"
    # chunk sizes of every rank (they may differ by a token or more)
    n = torch.tensor([k.shape[0]], dtype=torch.long, device=k.device if nccl else "cpu")
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(x) for x in sizes]
    q_max = int(q_pos.max()) if q_pos.numel() else -1
    cur = [k.contiguous(), v.contiguous(), k_pos.to(torch.long).to(k.device).contiguous()]
    for step in range(1, world):
        src = (rank - step) % world                 # owner of the chunk arriving this step
        m = sizes[src]
        bufs = [torch.empty((m,) + tuple(k.shape[1:]), dtype=k.dtype, device=k.device),
                torch.empty((m,) + tuple(v.shape[1:]), dtype=v.dtype, device=v.device),
                torch.empty(m, dtype=torch.long, device=k.device)]
        reqs = _exchange(cur, bufs, nxt, prv, nccl)
        if step > 1:
            # the chunk received in the previous step was sent on above; attend to it now,
            # while that transfer is in flight
            if not (causal and held_min > q_max):
                o2, l2 = attention_partial(q, held[0], held[1], q_pos, held[2], scale, causal, window, softcap,
                                           alibi)
                o, lse = merge_partials(o, lse, o2, l2)
        for r in reqs:
            r.wait()
        held = bufs
        held_min = int(bufs[2].min()) if m else 1 << 62
        cur = bufs
    if not (causal and held_min > q_max):
        o2, l2 = attention_partial(q, held[0], held[1], q_pos, held[2], scale, causal, window, softcap, alibi)
        o, lse = merge_partials(o, lse, o2, l2)
    return o.to(q.dtype)
