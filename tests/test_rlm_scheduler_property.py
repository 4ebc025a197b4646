"""Random operation sequences on the RLM call-tree scheduler (CPU): spawns, starts,
completions, failures, cancellations and timeouts in random order.  Invariants: a call
in a terminal state never changes again; below a failed, cancelled or timed-out call
nothing is pending or running (spawning anywhere under one yields a cancelled call); ready()
never exceeds the per-level concurrency; the depth limit holds."""
import random

import pytest

from rusteeze_b200.rlm.recursive_scheduler import CallState, RecursiveScheduler, SchedulerLimits

TERMINAL = {CallState.DONE, CallState.FAILED, CallState.CANCELLED, CallState.TIMED_OUT}
DEAD = {CallState.FAILED, CallState.CANCELLED, CallState.TIMED_OUT}


def _descendants(s, cid):
    out, todo = [], list(s.nodes[cid].children)
    while todo:
        c = todo.pop()
        out.append(c)
        todo.extend(s.nodes[c].children)
    return out


def _ancestors(s, cid):
    out, p = [], s.nodes[cid].parent
    while p is not None:
        out.append(p)
        p = s.nodes[p].parent
    return out


@pytest.mark.parametrize("seed", range(40))
def test_random_call_trees_keep_their_invariants(seed):
    rng = random.Random(seed)
    lim = SchedulerLimits(max_depth=3, per_level_concurrency=rng.randint(1, 3), max_pending=60, call_timeout_s=10.0)
    s = RecursiveScheduler(lim)
    final = {}
    for _ in range(300):
        ids = [c for c in s.nodes if c != 0]
        op = rng.random()
        if op < 0.3 or not ids:
            parent = rng.choice([0] + ids)
            if s.nodes[parent].depth < lim.max_depth and s.num_pending() < lim.max_pending:
                c = s.spawn(parent, "p", "i")
                if any(s.nodes[a].state in DEAD for a in _ancestors(s, c)):
                    assert s.nodes[c].state == CallState.CANCELLED
        elif op < 0.5:
            ready = s.ready()
            depths = {}
            for n in s.nodes.values():
                if n.state == CallState.RUNNING:
                    depths[n.depth] = depths.get(n.depth, 0) + 1
            for n in ready:
                depths[n.depth] = depths.get(n.depth, 0) + 1
            assert all(v <= lim.per_level_concurrency for d, v in depths.items() if d > 0)
            if ready:
                s.start(rng.choice(ready).call_id)
        elif op < 0.65:
            s.complete(rng.choice(ids), "ok")
        elif op < 0.75:
            s.fail(rng.choice(ids), "boom")
        elif op < 0.85:
            s.cancel(rng.choice(ids))
        else:
            running = [c for c in ids if s.nodes[c].state == CallState.RUNNING]
            if running:
                s.check_timeouts(now=s.nodes[rng.choice(running)].started + 1e6)
        for cid, n in s.nodes.items():
            if cid in final:
                assert n.state == final[cid], f"call {cid} left terminal state {final[cid]} for {n.state}"
            elif n.state in TERMINAL:
                final[cid] = n.state
            if n.state in DEAD:
                for d in _descendants(s, cid):
                    assert s.nodes[d].state not in (CallState.PENDING, CallState.RUNNING), (cid, d)
            assert n.depth <= lim.max_depth
