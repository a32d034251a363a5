"""Prefix cache (prefixSnapshot, cmd/monolith/monolith.go:5868-5952) over the
engine simulator on the CPU oracle.

The snapshot only moves K/V rows, bit for bit, so an engine with the prefix
cache must produce exactly the outputs of one without it, while admitting later
requests with their shared prefix already in place (restore, M:5881-5905) and
offering finished sessions' positions back (capture, M:5927-5952).
"""

import numpy as np
import pytest

from engine_sim import simulate


def _model(oracle, pt=16):
    cfg = oracle.make_config(300, 64, 96, 2, 4, 2, 256, rope_theta=1e5, tied=True, weight_format="q8",
                             page_tokens=pt)
    m = oracle.Model(cfg)
    m.init_synthetic(17, 0.02)
    return m


def _requests(seed, n=6, system=40):
    rng = np.random.default_rng(seed)
    head = rng.integers(0, 300, size=system).tolist()
    reqs = []
    for i in range(n):
        tail = rng.integers(0, 300, size=int(rng.integers(1, 9))).tolist()
        r = dict(ids=head + tail, max_tokens=int(rng.integers(2, 6)), seed=50 + i)
        if i % 2:
            r.update(temperature=0.7, top_k=20, top_p=0.9, penalty=1.1)
        reqs.append(r)
    return reqs


@pytest.mark.parametrize("tail", [False, True])
def test_prefix_cache_keeps_outputs_and_reuses_prefix(oracle, tail):
    m = _model(oracle)
    reqs = _requests(3)
    # max_batch 1: each request is admitted after the previous one finished and
    # offered its positions to the snapshot.
    base, _ = simulate(m, reqs, 16, 1, 16, 8, 1)
    st = {}
    got, trace = simulate(m, reqs, 16, 1, 16, 8, 1, prefix_limit=4, prefix_tail=tail, stats=st)
    assert got == base
    # every request after the first matches at least the 40-token system prompt
    assert st["prefix_hits"] == len(reqs) - 1
    pt = m.cfg.page_tokens
    assert st["prefix_tokens"] >= (len(reqs) - 1) * (40 // pt) * pt
    if tail:
        assert st["prefix_tokens"] >= (len(reqs) - 1) * 40
    # borrowed snapshot pages (ids >= limit) appear in later page tables
    assert any(p >= 16 for _, tables, _ in trace for t in tables for p in t)


def test_prefix_cache_with_concurrent_borrowers(oracle):
    """Several sessions borrow the snapshot at once; capture is skipped while
    another session borrows it (M:5928-5931) and outputs stay unchanged."""
    m = _model(oracle)
    reqs = _requests(8, n=7)
    base, _ = simulate(m, reqs, 24, 3, 24, 8, 2)
    st = {}
    got, _ = simulate(m, reqs, 24, 3, 24, 8, 2, prefix_limit=3, prefix_tail=True, stats=st)
    assert got == base
    assert st["prefix_hits"] >= 3


def test_prefix_limit_caps_snapshot_pages(oracle):
    """A snapshot keeps at most prefix_limit pages (capture's n, M:5936-5938):
    with one page only the first page_tokens positions are ever restored."""
    m = _model(oracle)
    reqs = _requests(4)
    base, _ = simulate(m, reqs, 16, 1, 16, 8, 1)
    st = {}
    got, _ = simulate(m, reqs, 16, 1, 16, 8, 1, prefix_limit=1, prefix_tail=True, stats=st)
    assert got == base
    assert st["prefix_pages"] == 1
    assert st["prefix_tokens"] == (len(reqs) - 1) * m.cfg.page_tokens


def test_prefix_cache_random_scenarios(oracle):
    """Seeded random request mixes (several shared system prompts, random
    suffixes, output lengths, batch sizes, snapshot limits, tail reuse): the
    simulated engine with the prefix cache always returns exactly the outputs
    of the engine without it, and never reuses more tokens than a prompt holds."""
    m = _model(oracle)
    rng = np.random.default_rng(77)
    for scenario in range(5):
        heads = [rng.integers(0, 300, size=int(rng.integers(10, 50))).tolist() for _ in range(2)]
        reqs = []
        for i in range(int(rng.integers(3, 7))):
            head = heads[int(rng.integers(0, 2))]
            tail = rng.integers(0, 300, size=int(rng.integers(1, 10))).tolist()
            r = dict(ids=head + tail, max_tokens=int(rng.integers(1, 5)), seed=int(rng.integers(1, 1000)))
            if rng.random() < 0.5:
                r.update(temperature=0.9, top_k=30, top_p=0.9, penalty=1.05)
            reqs.append(r)
        mb = int(rng.integers(1, 4))
        limit, plimit, tail = 28, int(rng.integers(1, 5)), bool(rng.random() < 0.5)
        base, _ = simulate(m, reqs, limit, mb, 16, 8, 1)
        st = {}
        got, _ = simulate(m, reqs, limit, mb, 16, 8, 1, prefix_limit=plimit, prefix_tail=tail, stats=st)
        assert got == base, scenario
        assert st["prefix_tokens"] <= sum(len(r["ids"]) - 1 for r in reqs)
        assert st["prefix_pages"] <= plimit
