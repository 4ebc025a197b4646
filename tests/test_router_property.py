"""Replica router properties under random operation sequences, and the data-parallel
serving front end (two CPU engine replicas behind the router) through the HTTP app."""
import asyncio
import collections
import json
import random

import pytest
from fastapi.testclient import TestClient

from rusteeze_b200.engine.router import LatencyHistogram, Policy, Replica, ReplicaRouter

_SEEDS = range(12)


@pytest.mark.parametrize("policy", list(Policy))
@pytest.mark.parametrize("seed", _SEEDS)
def test_random_select_release_health_sequences(policy, seed):
    """Invariants over a random mix of select / release / health flips:
    a down replica is never picked, in-flight counts equal the picks not yet released,
    least-loaded picks a minimum-load live replica, and `served` counts releases."""
    rng = random.Random(seed)
    n = rng.randint(1, 5)
    reps = [Replica(f"r{i}", None) for i in range(n)]
    rt = ReplicaRouter(reps, policy, seed=seed)
    held = collections.Counter()
    released = collections.Counter()
    for _ in range(400):
        op = rng.random()
        if op < 0.5:
            live = [r for r in reps if r.healthy]
            if not live:
                with pytest.raises(RuntimeError):
                    rt.select()
                continue
            before = {r.name: r.in_flight for r in reps}
            r = rt.select()
            assert r.healthy
            if policy == Policy.LEAST_LOADED:
                assert before[r.name] == min(before[x.name] for x in live)
            held[r.name] += 1
        elif op < 0.85:
            busy = [r for r in reps if held[r.name] > 0]
            if busy:
                r = rng.choice(busy)
                rt.release(r, latency_s=rng.random() * 0.1, error=rng.random() < 0.1)
                held[r.name] -= 1
                released[r.name] += 1
        else:
            rt.set_health(rng.choice(reps).name, rng.random() < 0.6)
        for r in reps:
            assert r.in_flight == held[r.name] >= 0
            assert r.served == released[r.name]
            assert r.errors <= r.served


def test_round_robin_is_fair_over_a_fixed_live_set():
    reps = [Replica(f"r{i}", None) for i in range(4)]
    rt = ReplicaRouter(reps, Policy.ROUND_ROBIN)
    rt.set_health("r2", False)
    picks = collections.Counter(rt.select().name for _ in range(300))
    assert picks == {"r0": 100, "r1": 100, "r3": 100}


def test_least_loaded_balances_a_steady_stream():
    """With every request released after a fixed number of later arrivals, least-loaded
    keeps the replicas' served counts within one of each other."""
    reps = [Replica(f"r{i}", None) for i in range(3)]
    rt = ReplicaRouter(reps)
    window = collections.deque()
    for _ in range(301):
        window.append(rt.select())
        if len(window) > 5:
            rt.release(window.popleft())
    served = [r.served for r in reps]
    assert max(served) - min(served) <= 1


def test_prefix_affinity_is_sticky_balanced_and_moves_only_a_dead_replica_s_keys():
    from rusteeze_b200.engine.router import AFFINITY_SLACK, affinity_key
    reps = [Replica(f"dp{i}", None) for i in range(4)]
    r = ReplicaRouter(reps, Policy.PREFIX_AFFINITY)
    keys = [affinity_key(list(range(i, i + 300))) for i in range(400)]
    first = {}
    for k in keys:
        x = r.select(k)
        r.release(x)
        first[k] = x.name
        y = r.select(k)                           # the same prompt opening: the same replica
        r.release(y)
        assert y.name == x.name
    spread = collections.Counter(first.values())
    assert len(spread) == 4 and min(spread.values()) > 400 / 4 * 0.6, spread
    # only tokens past AFFINITY_TOKENS differ: same key
    assert affinity_key(list(range(300)) + [1]) == affinity_key(list(range(300)) + [2])
    assert affinity_key(prompt="a system prompt") == affinity_key(prompt="a system prompt")
    r.set_health("dp2", False)
    for k in keys:
        x = r.select(k)
        r.release(x)
        if first[k] != "dp2":
            assert x.name == first[k]             # keys of live replicas stay put
        else:
            assert x.name != "dp2"
    # load guard: a hot key spills to the least-loaded replica
    r.set_health("dp2", True)
    k = keys[0]
    held = [r.select(k) for _ in range(AFFINITY_SLACK)]
    assert all(h.name == first[k] for h in held)
    spill = r.select(k)
    assert spill.name != first[k]


def test_unknown_replica_name_is_an_error():
    rt = ReplicaRouter([Replica("a", None)])
    with pytest.raises(KeyError):
        rt.set_health("b", False)


@pytest.mark.parametrize("seed", range(6))
def test_latency_percentiles_bound_the_samples(seed):
    """The p-th percentile is the midpoint of the log2 bucket holding the sample of rank
    ceil(p/100 * n): within a factor 1.5 of that sample."""
    rng = random.Random(seed)
    xs = [10 ** rng.uniform(-5, 1) for _ in range(rng.randint(1, 300))]
    h = LatencyHistogram()
    for x in xs:
        h.record(x)
    s = sorted(xs)
    for q in (0, 1, 50, 90, 99, 100):
        import math
        k = max(1, math.ceil(q / 100 * len(s)))
        v = max(s[k - 1], 1e-6)
        p = h.percentile(q)
        assert v / 1.5 <= p <= v * 1.5 + 1e-12, (q, v, p)


# ----------------------------------------------------------------------------- DP front end
def _cfg(dp=2):
    from rusteeze_b200.config.config import Config
    cfg = Config()
    cfg.model.preset = "tiny-llama"
    cfg.model.device = "cpu"
    cfg.model.dtype = "float32"
    cfg.model.data_parallel_size = dp
    cfg.engine.num_gpu_blocks = 64
    cfg.engine.max_num_seqs = 4
    cfg.engine.max_num_batched_tokens = 256
    cfg.logging.request_logging = False
    return cfg


@pytest.fixture()
def dp_app():
    from rusteeze_b200.api.server import create_app
    from rusteeze_b200.engine.dp_engine import ReplicatedAsyncEngine
    cfg = _cfg()
    front = ReplicatedAsyncEngine.from_config(cfg).start()
    yield TestClient(create_app(front, cfg)), front
    front.shutdown()


def test_replicas_get_identical_weights_and_one_config_each():
    from rusteeze_b200.config.validation import collect_errors
    from rusteeze_b200.engine.dp_engine import replica_configs
    cfg = _cfg(3)
    assert not collect_errors(cfg)
    cs = replica_configs(cfg)
    assert [c.model.device for c in cs] == ["cpu"] * 3
    assert all(c.model.data_parallel_size == 1 and c.model.tensor_parallel_size == 1 for c in cs)
    assert cfg.model.data_parallel_size == 3           # the caller's config is left alone
    bad = _cfg(2)
    bad.model.tensor_parallel_size = 2
    assert any("data_parallel_size" in e for e in collect_errors(bad))


def test_dp_front_end_spreads_requests_and_every_replica_answers_alike(dp_app):
    c, front = dp_app
    import concurrent.futures as cf
    body = {"prompt": "the same prompt", "max_tokens": 6, "temperature": 0, "ignore_eos": True}
    with cf.ThreadPoolExecutor(8) as ex:
        rs = list(ex.map(lambda _: c.post("/v1/completions", json=body), range(16)))
    assert all(r.status_code == 200 for r in rs), [r.text for r in rs if r.status_code != 200]
    texts = {r.json()["choices"][0]["text"] for r in rs}
    assert len(texts) == 1                               # greedy, same weights on every replica
    st = front.stats()
    served = [r["served"] for r in st["replicas"]]
    assert sum(served) == 16 and min(served) >= 1, served
    assert all(r["in_flight"] == 0 for r in st["replicas"])
    assert st["requests_processed"] == 16 and st["data_parallel_size"] == 2
    text = c.get("/metrics").text
    line = [ln for ln in text.splitlines() if ln.startswith("rusteeze_inference_generation_tokens_total")][0]
    assert float(line.split()[-1]) == 16 * 6             # every replica's steps reach the metrics
    h = c.get("/health").json()
    assert h["status"] == "healthy"


def test_dp_stream_and_abort_reach_the_owning_replica(dp_app):
    c, front = dp_app
    with c.stream("POST", "/v1/completions", json={"prompt": "abc", "max_tokens": 5, "stream": True,
                                                   "temperature": 0, "ignore_eos": True}) as r:
        lines = [ln for ln in r.iter_lines() if ln]
    assert lines[-1] == "data: [DONE]"
    assert sum(len(json.loads(x[6:])["choices"][0]["text"]) >= 0 for x in lines[:-1]) >= 1

    async def abort_midway():
        from rusteeze_b200.core.sampling_params import SamplingParams
        agen = front.generate("xyz", SamplingParams(max_tokens=200, ignore_eos=True), "rid-abort")
        first = await agen.__anext__()
        owner = front._owner["rid-abort"]
        front.abort("rid-abort")
        outs = [first]
        async for o in agen:
            outs.append(o)
        return owner, outs
    owner, outs = asyncio.run(abort_midway())
    assert outs[-1].finished and len(outs) < 200
    assert owner.in_flight == 0 and "rid-abort" not in front._owner


def test_a_failed_replica_is_routed_around(dp_app):
    c, front = dp_app
    bad = front.replicas[1]

    def boom():
        raise RuntimeError("injected step failure")
    bad.engine.step = boom
    codes = [c.post("/v1/completions", json={"prompt": f"p{i}", "max_tokens": 3, "ignore_eos": True}).status_code
             for i in range(8)]
    # at most the request that found replica 1 still marked ready fails; the rest go to replica 0
    assert codes.count(503) <= 1 and codes.count(200) >= 7, codes
    st = {r["name"]: r for r in front.stats()["replicas"]}
    assert st["dp1"]["healthy"] is False and st["dp0"]["healthy"] is True
    assert st["dp1"]["errors"] == codes.count(503)
    assert c.get("/health/ready").status_code == 200     # one replica still serves
    front.replicas[0].healthy = False
    assert c.post("/v1/completions", json={"prompt": "x", "max_tokens": 2}).status_code == 503
    assert c.get("/health/ready").status_code == 503


def test_dp_prefix_affinity_keeps_a_shared_prefix_on_one_replica():
    """Two CPU replicas with prefix caching: requests that share a long opening all reach
    the same replica, whose prefix cache serves the shared blocks."""
    from rusteeze_b200.core.sampling_params import SamplingParams
    from rusteeze_b200.engine.dp_engine import ReplicatedAsyncEngine
    cfg = _cfg()
    cfg.engine.enable_prefix_caching = True
    cfg.server.router_policy = "prefix_affinity"
    front = ReplicatedAsyncEngine.from_config(cfg).start()
    system = list(range(100, 400))                       # 300 shared tokens
    sp = SamplingParams(temperature=0.0, max_tokens=2, ignore_eos=True)

    async def run():
        for i in range(6):
            async for _ in front.generate(None, sp, f"r{i}", system + [7, i]):
                pass

    try:
        asyncio.run(run())
        served = sorted(r["served"] for r in front.stats()["replicas"])
        assert served == [0, 6], served
        hits = [ae.engine.bm.stats()["prefix_block_hits"] for ae in front.replicas]
        assert max(hits) >= 5 * (300 // 16)
    finally:
        front.shutdown()


def test_dp_front_end_serves_embeddings_and_the_tokenizer_endpoints(dp_app):
    c, front = dp_app
    r = c.post("/v1/embeddings", json={"input": [[5, 6, 7], [8, 9]]})
    assert r.status_code == 200, r.text
    import numpy as np
    want = front.replicas[0].engine.embed([[5, 6, 7]])[0]
    assert np.abs(np.array(r.json()["data"][0]["embedding"]) - want).max() < 1e-5
    t = c.post("/tokenize", json={"prompt": "hello"})
    assert t.status_code == 200 and t.json()["count"] > 0
    d = c.post("/detokenize", json={"tokens": t.json()["tokens"]})
    assert d.status_code == 200 and "hello" in d.json()["prompt"]
