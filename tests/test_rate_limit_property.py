"""Sliding-window rate limiter (CPU), random request times: within any 60 s window no
key gets more than per_minute + burst admissions, a key that waited a full window is
admitted again, and idle keys do not accumulate (a server keyed by client address sees
unboundedly many keys)."""
import random

import pytest

from rusteeze_b200.api.middleware import SlidingWindowLimiter


@pytest.mark.parametrize("seed", range(20))
def test_window_bound_and_recovery(seed):
    rng = random.Random(seed)
    per_min, burst = rng.randint(1, 8), rng.randint(0, 3)
    lim = SlidingWindowLimiter(per_min, burst)
    t, admitted = 0.0, {k: [] for k in "abc"}
    for _ in range(2000):
        t += rng.expovariate(2.0)
        k = rng.choice("abc")
        ok, limit, remaining, reset = lim.check(k, now=t)
        assert limit == per_min + burst and remaining >= 0 and reset >= 0
        if ok:
            admitted[k].append(t)
    for k, ts in admitted.items():
        j = 0
        for i, x in enumerate(ts):               # every 60 s window [x, x+60)
            while j < len(ts) and ts[j] < x + 60.0:
                j += 1
            assert j - i <= per_min + burst
    assert lim.check("a", now=t + 61.0)[0]       # a full idle window later: admitted again


def test_idle_keys_are_forgotten():
    lim = SlidingWindowLimiter(5)
    for i in range(10_000):
        lim.check(f"client-{i}", now=float(i % 50))
    for j in range(1100):                       # later traffic from one client; the others are idle
        lim.check("late", now=10_000.0 + j)
    assert len(lim.hits) <= 64
