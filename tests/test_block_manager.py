"""Block manager: C++ implementation vs the Python mirror under random
operation sequences (refcount conservation, no double free, CoW, swap,
prefix-cache accounting), plus the reference's seed scenarios
(crates/rusteeze-engine/src/block_manager.rs:250-294)."""
import numpy as np
from hypothesis import given, settings, strategies as st

from rusteeze_b200.engine.block_manager import PyBlockManager, make_block_manager


def test_allocate_free_fork_swap_basic():
    bm = make_block_manager(16, 8, 8, True)
    t = np.arange(40, dtype=np.int64)
    assert bm.allocate_prompt(1, t) == 0
    bm.ensure_capacity(1, 40, 0)
    assert len(bm.block_table(1)) == 3 and bm.num_free_gpu_blocks() == 5
    bm.fork(1, 2)
    assert all(bm.ref_count(b) == 2 for b in bm.block_table(1))
    cow = bm.ensure_capacity(2, 41, 40)        # writes into the shared 3rd block -> copy
    assert len(cow) == 1 and cow[0][0] == bm.block_table(1)[2]
    m = bm.swap_out(2)
    assert len(m) == 3 and bm.can_swap_in(2)
    m2 = bm.swap_in(2)
    assert len(m2) == 3
    bm.free(1)
    bm.free(2)
    assert bm.check_invariants() and bm.num_free_gpu_blocks() == 8


def test_prefix_cache_chain_and_eviction():
    bm = make_block_manager(16, 6, 0, True)
    a = np.arange(64, dtype=np.int64)
    bm.allocate_prompt(1, a)
    bm.ensure_capacity(1, 64, 0)
    bm.commit(1, a, 64)
    bm.free(1)
    assert bm.num_cached_free_blocks() == 4
    b = np.concatenate([a[:48], np.arange(1000, 1020)]).astype(np.int64)
    assert bm.cached_prefix_len(b) == 48        # 3 shared leading blocks
    c = a.copy()
    c[5] = 99                                   # differs in block 0 -> no reuse at all
    assert bm.cached_prefix_len(c) == 0
    # exhausting the free list evicts cached blocks (LRU)
    bm.allocate_prompt(2, np.arange(5000, 5096, dtype=np.int64))
    bm.ensure_capacity(2, 96, 0)
    assert bm.stats()["evictions"] >= 4 and bm.check_invariants()


OPS = st.lists(st.tuples(st.sampled_from(["new", "grow", "fork", "free", "swap_out", "swap_in", "commit"]),
                         st.integers(0, 7), st.integers(1, 70)), min_size=1, max_size=60)


@settings(max_examples=60, deadline=None)
@given(OPS, st.booleans())
def test_cpp_matches_python_mirror(ops, prefix):
    cpp = make_block_manager(16, 24, 12, prefix)
    py = PyBlockManager(16, 24, 12, prefix)
    toks = {}
    on_cpu = set()
    rng = np.random.default_rng(0)
    next_id = [100]
    for kind, k, n in ops:
        ids = sorted(toks)
        if kind == "new":
            sid = next_id[0]
            next_id[0] += 1
            t = rng.integers(0, 4, n).astype(np.int64)     # tiny alphabet -> frequent prefix hits
            need = -(-n // 16)
            if need > py.num_free_gpu_blocks():
                continue
            assert cpp.allocate_prompt(sid, t) == py.allocate_prompt(sid, t)
            toks[sid] = t
            assert cpp.ensure_capacity(sid, n, 0) == py.ensure_capacity(sid, n, 0)
        elif not ids:
            continue
        else:
            sid = ids[k % len(ids)]
            if kind == "grow" and sid not in on_cpu:
                cur = len(toks[sid])
                new_len = cur + n % 20 + 1
                if cpp.blocks_to_grow(sid, new_len, cur) != py.blocks_to_grow(sid, new_len, cur):
                    raise AssertionError("blocks_to_grow differs")
                if py.blocks_to_grow(sid, new_len, cur) > py.num_free_gpu_blocks():
                    continue
                assert cpp.ensure_capacity(sid, new_len, cur) == py.ensure_capacity(sid, new_len, cur)
                toks[sid] = np.concatenate([toks[sid], rng.integers(0, 4, new_len - cur)]).astype(np.int64)
            elif kind == "commit" and sid not in on_cpu:
                cpp.commit(sid, toks[sid], len(toks[sid]))
                py.commit(sid, toks[sid], len(toks[sid]))
            elif kind == "fork" and sid not in on_cpu:
                c = next_id[0]
                next_id[0] += 1
                cpp.fork(sid, c)
                py.fork(sid, c)
                toks[c] = toks[sid].copy()
            elif kind == "free":
                cpp.free(sid)
                py.free(sid)
                del toks[sid]
                on_cpu.discard(sid)
            elif kind == "swap_out" and sid not in on_cpu:
                if not py.can_swap_out(sid):
                    continue
                assert cpp.swap_out(sid) == py.swap_out(sid)
                on_cpu.add(sid)
            elif kind == "swap_in" and sid in on_cpu:
                if len(py.block_table(sid)) > py.num_free_gpu_blocks():
                    continue
                assert cpp.swap_in(sid) == py.swap_in(sid)
                on_cpu.discard(sid)
        assert cpp.num_free_gpu_blocks() == py.num_free_gpu_blocks()
        assert cpp.num_free_cpu_blocks() == py.num_free_cpu_blocks()
        for s in toks:
            assert cpp.block_table(s) == py.block_table(s)
        assert cpp.check_invariants()
    for s in list(toks):
        cpp.free(s)
    assert cpp.check_invariants() and cpp.num_free_gpu_blocks() == 24


def test_batch_builder_layout():
    import torch
    bm = make_block_manager(16, 32, 0, False)
    seqs = {1: np.arange(20, dtype=np.int64), 2: np.arange(100, 105, dtype=np.int64)}
    for s, t in seqs.items():
        bm.allocate_prompt(s, t)
        bm.ensure_capacity(s, len(t) + 1, 0)
    T, S, MB = 64, 2, 8
    bufs = {k: torch.zeros(n, dtype=dt) for k, n, dt in [
        ("ids", T, torch.int64), ("pos", T, torch.int64), ("slot", T, torch.int64), ("qsl", S + 1, torch.int32),
        ("sl", S, torch.int32), ("bt", S * MB, torch.int32), ("li", T, torch.int64)]}
    # seq 1: decode of its 21st token (ctx 20, 1 new); seq 2: full 5-token prefill
    n = bm.build_batch(np.array([1, 2]), np.array([20, 0]), np.array([1, 5]),
                       np.array([7, 100, 101, 102, 103, 104], dtype=np.int64),
                       *(bufs[k].data_ptr() for k in ("ids", "pos", "slot", "qsl", "sl", "bt", "li")), MB, 1)
    assert n == 6
    assert bufs["qsl"].tolist() == [0, 1, 6] and bufs["sl"].tolist() == [21, 5]
    assert bufs["pos"][:6].tolist() == [20, 0, 1, 2, 3, 4]
    b1 = bm.block_table(1)
    assert bufs["slot"][0].item() == b1[1] * 16 + 4
    assert bufs["li"][:2].tolist() == [0, 5]
