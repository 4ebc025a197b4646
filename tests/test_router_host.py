"""Replica router policies and the C++ host runtime pieces (size-class pool,
shared-memory broadcast ring across processes, NUMA helpers)."""
import multiprocessing as mp
import os

import pytest

from rusteeze_b200.engine.router import LatencyHistogram, Policy, Replica, ReplicaRouter


def test_least_loaded_and_health():
    rs = [Replica(f"r{i}", None) for i in range(3)]
    rt = ReplicaRouter(rs, Policy.LEAST_LOADED)
    a, b, c = rt.select(), rt.select(), rt.select()
    assert {a.name, b.name, c.name} == {"r0", "r1", "r2"}
    rt.release(a, 0.01)
    assert rt.select() is a
    rt.set_health("r1", False)
    for _ in range(10):
        assert rt.select().name != "r1"


def test_round_robin_random_and_prober():
    rs = [Replica(f"r{i}", None) for i in range(3)]
    rt = ReplicaRouter(rs, Policy.ROUND_ROBIN)
    assert [rt.select().name for _ in range(4)] == ["r0", "r1", "r2", "r0"]
    rt2 = ReplicaRouter(rs, Policy.RANDOM, prober=lambda r: r.name != "r2")
    rt2.probe()
    assert all(rt2.select().name != "r2" for _ in range(20))
    rt3 = ReplicaRouter([Replica("x", None)], prober=lambda r: 1 / 0)
    rt3.probe()
    with pytest.raises(RuntimeError):
        rt3.select()


def test_latency_histogram():
    h = LatencyHistogram()
    for i in range(100):
        h.record(0.001 if i < 90 else 0.5)
    assert h.percentile(50) < 0.003 and h.percentile(99) > 0.2


def test_size_class_pool():
    from rusteeze_b200._host import SizeClassPool
    p = SizeClassPool()
    a = p.acquire(1000)
    p.release(a, 1000)
    b = p.acquire(900)          # same 1 KiB class -> reused
    assert a == b and p.stats()["hits"] == 1
    assert SizeClassPool.size_class(300) == 512


def _reader(name, idx, n, q):
    from rusteeze_b200._host import ShmRing
    r = ShmRing(name, False)
    got = []
    for _ in range(n):
        m = r.consume(idx, 10.0)
        got.append(m)
    q.put((idx, got))


def test_shm_ring_broadcast_two_readers():
    from rusteeze_b200._host import ShmRing
    name = f"/rz_test_{os.getpid()}"
    w = ShmRing(name, True, 2, 1024, 2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_reader, args=(name, i, 5, q)) for i in range(2)]
    for p in ps:
        p.start()
    for i in range(5):                     # ring of 2 slots: publish blocks until both read
        assert w.publish(f"msg{i}".encode(), 10.0)
    res = dict(q.get(timeout=30) for _ in range(2))
    for p in ps:
        p.join(10)
    assert res[0] == res[1] == [f"msg{i}".encode() for i in range(5)]


def test_shm_ring_timeout_and_close():
    from rusteeze_b200._host import ShmRing
    w = ShmRing(f"/rz_test2_{os.getpid()}", True, 1, 64, 1)
    assert w.publish(b"a", 0.1)
    assert not w.publish(b"b", 0.2)       # nobody consumed slot 0: bounded wait gives up
    r = ShmRing(f"/rz_test2_{os.getpid()}", False)
    assert r.consume(0, 0.1) == b"a"
    assert r.consume(0, 0.1) is None       # nothing new -> timeout
    w.close()
    assert r.closed


def test_numa_helpers():
    from rusteeze_b200 import _host as H
    assert H.numa_num_nodes() >= 1
    cpus = H.numa_node_cpus(0)
    assert len(cpus) >= 1
    aff = H.get_affinity()
    assert H.set_affinity(aff[:1]) and H.get_affinity() == aff[:1]
    H.set_affinity(aff)
    assert H.pci_numa_node("0000:ff:ff.7") == -1
