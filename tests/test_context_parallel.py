"""Context-parallel ring attention on gloo ranks: every rank's output rows equal the dense
oracle on the whole sequence, for zigzag and contiguous splits, GQA, sliding windows,
soft-caps and ALiBi; plus the pieces (split, partial attention, log-sum-exp merge) alone."""
import os
import socket

import pytest
import torch

from rusteeze_b200.ops import reference as ref
from rusteeze_b200.parallel import context_parallel as cp


def _dense(q, k, v, scale, window=None, softcap=None, alibi=None):
    T = q.shape[0]
    qsl = torch.tensor([0, T], dtype=torch.int32)
    # the paged oracle over one sequence whose cache holds k / v in 16-token blocks
    nb = (T + 15) // 16
    kc = torch.zeros(nb * 16, k.shape[1], k.shape[2])
    vc = torch.zeros_like(kc)
    kc[:T], vc[:T] = k, v
    kc = kc.view(nb, 16, k.shape[1], k.shape[2]).permute(0, 2, 1, 3).contiguous()
    vc = vc.view(nb, 16, v.shape[1], v.shape[2]).permute(0, 2, 1, 3).contiguous()
    bt = torch.arange(nb, dtype=torch.int32).view(1, -1)
    return ref.paged_attention(q, kc, vc, qsl, torch.tensor([T], dtype=torch.int32), bt, scale, window, softcap,
                               alibi)


def test_zigzag_split_covers_the_sequence_once():
    for T, W in ((10, 2), (1000, 4), (37, 8), (5, 4)):
        parts = cp.zigzag_split(T, W)
        pos = torch.cat([cp.positions_of(p) for p in parts])
        assert sorted(pos.tolist()) == list(range(T))
        sizes = [sum(b - a for a, b in p) for p in parts]
        assert max(sizes) - min(sizes) <= 2


def test_partials_merge_to_the_full_attention():
    g = torch.Generator().manual_seed(0)
    T, H, D = 40, 4, 16
    q, k, v = (torch.randn(T, H, D, generator=g) for _ in range(3))
    pos = torch.arange(T)
    full, _ = cp.attention_partial(q, k, v, pos, pos, D ** -0.5)
    o1, l1 = cp.attention_partial(q, k[:13], v[:13], pos, pos[:13], D ** -0.5)
    o2, l2 = cp.attention_partial(q, k[13:], v[13:], pos, pos[13:], D ** -0.5)
    o, _ = cp.merge_partials(o1, l1, o2, l2)
    assert torch.allclose(o, full, atol=1e-5)
    assert torch.allclose(full, _dense(q, k, v, D ** -0.5), atol=1e-5)
    # a query that sees no key of a chunk (lse -inf) takes the other chunk as is
    assert torch.isinf(l2[:13]).all()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q_out, split, kw):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(1)
        T, Hq, Hkv, D = 203, 8, 2, 32
        q = torch.randn(T, Hq, D, generator=g)
        k = torch.randn(T, Hkv, D, generator=g)
        v = torch.randn(T, Hkv, D, generator=g)
        alibi = ref.alibi_slopes(Hq) if kw.get("alibi") else None
        want = _dense(q, k, v, D ** -0.5, kw.get("window"), kw.get("softcap"), alibi)
        if split == "zigzag":
            ranges = cp.zigzag_split(T, world)[rank]
        else:
            per = -(-T // world)
            ranges = [(rank * per, min(T, (rank + 1) * per))]
        pos = cp.positions_of(ranges)
        got = cp.ring_attention(q[pos], k[pos], v[pos], pos, pos, D ** -0.5, window=kw.get("window"),
                                softcap=kw.get("softcap"), alibi=alibi)
        q_out.put((rank, float((got - want[pos]).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("split,kw", [("zigzag", {}), ("contiguous", {}), ("zigzag", {"window": 50}),
                                      ("zigzag", {"softcap": 20.0, "alibi": True})])
def test_ring_attention_matches_the_dense_oracle(world, split, kw):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, split, kw)) for r in range(world)]
    for p in ps:
        p.start()
    errs = dict(q.get(timeout=240) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in ps)
    assert max(errs.values()) < 1e-4, errs
