"""GPU parity: libsrstep.so (through its C ABI) against the CPU oracle.

SR_MODE_EXACT reproduces the reference's operation order, so logits, K/V rows,
greedy ids and sampled ids are compared bit for bit with the oracle; the
Transformers goldens are also checked at the reference's 2e-5.
"""

import ctypes as C

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _step_mod():
    from sr_go_tranformer_b200 import step
    return step


def device_from_oracle(om, srlib, mode="exact"):
    S = _step_mod()
    c = om.cfg
    d = S.make_desc(c.vocab, c.dim, c.hidden, c.layers, c.heads, c.kv_heads, c.context, c.rope_theta, c.norm_eps,
                    bool(c.tied), bool(c.qkv_bias), {0: "f32", 1: "q8", 2: "q4", 3: "q4-mixed"}[c.weight_format],
                    c.page_tokens)
    if c.rope_scaling:
        d.rope_scaling, d.rope_factor = 1, c.rope_factor
        d.rope_low_freq_factor, d.rope_high_freq_factor = c.rope_low, c.rope_high
        d.rope_original_max_positions = c.rope_original
    dm = S.Model(d)
    for i in range(om.nparams):
        vals, sc = om.get_param_raw(i)
        dm.load_param(i, vals, sc)
    dm.set_mode(mode)
    return dm


def assert_same(a, b, what):
    a, b = np.asarray(a), np.asarray(b)
    if not np.array_equal(a, b, equal_nan=True):
        bad = np.argwhere(~((a == b) | (np.isnan(a) & np.isnan(b))))
        i = tuple(bad[0])
        raise AssertionError(f"{what}: {len(bad)} mismatches, first at {i}: {a[i]!r} vs {b[i]!r}, "
                             f"max abs {np.nanmax(np.abs(a.astype(np.float64) - b)):.3g}")


def compare_cache_rows(pool, opool, om, cache):
    """Every written (layer, position) K/V row of a cache equals the oracle's."""
    pt, kd, pe = om.cfg.page_tokens, om.cfg.dim // om.cfg.heads * om.cfg.kv_heads, om.page_elements
    for pos in range(cache.pos):
        pg, slot = cache.pages[pos // pt], pos % pt
        for layer in range(om.cfg.layers):
            k, v = pool.read_row(pg, layer, slot)
            base = pg * pe + layer * 2 * pt * kd + slot * kd
            assert_same(k, opool[base:base + kd], f"K pos {pos} layer {layer}")
            assert_same(v, opool[base + pt * kd:base + pt * kd + kd], f"V pos {pos} layer {layer}")


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.split("/")[-1][:-4])
def test_golden_fixture_exact(oracle, srlib, path):
    S = _step_mod()
    om, z, hf = oracle.load_golden(path)
    dm = device_from_oracle(om, srlib)
    ids, ref = z["ids"], z["logits"]
    pool = S.PagePool(dm, 4)
    opool = np.zeros(4 * om.page_elements, dtype=np.float32)
    for chunk in (1, 4, 16, 35):
        cache = dm.new_cache(pool)
        opool[:] = 0
        for lo in range(0, 35, chunk):
            hi = min(lo + chunk, 35)
            before = cache.pos
            got = dm.prefill_selected([cache], [ids[lo:hi]])
            want = om.step(opool, [before], [ids[lo:hi]], [cache.pages])
            assert_same(got, want, f"chunk {chunk} rows {lo}:{hi}")
            assert np.abs(got[0] - ref[hi - 1]).max() <= 2e-5
        for p in (35, 36):
            got = dm.step(cache, int(ids[p]))
            want = om.step(opool, [p], [ids[p:p + 1]], [cache.pages])
            assert_same(got, want[0], f"decode {p}")
            assert np.abs(got - ref[p]).max() <= 2e-5
        compare_cache_rows(pool, opool, om, cache)
        cache.close()


def synthetic_pair(oracle, srlib, fmt, pt, vocab=300, dim=64, hidden=96, layers=2, heads=4, kv_heads=2, context=256,
                   tied=True, bias=False, seed=11):
    cfg = oracle.make_config(vocab, dim, hidden, layers, heads, kv_heads, context, rope_theta=1e5, tied=tied,
                             qkv_bias=bias, weight_format=fmt, page_tokens=pt)
    om = oracle.Model(cfg)
    om.init_synthetic(seed, 0.02 if fmt != "f32" else 0.05)
    return om, device_from_oracle(om, srlib)


@pytest.mark.parametrize("pt", [16, 32])
@pytest.mark.parametrize("fmt,tied,bias", [("f32", True, False), ("q8", False, False), ("q4", True, True),
                                           ("q4-mixed", False, True)])
def test_ragged_mixed_batches_exact(oracle, srlib, fmt, tied, bias, pt):
    S = _step_mod()
    om, dm = synthetic_pair(oracle, srlib, fmt, pt, tied=tied, bias=bias)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, om.cfg.vocab, size=n).tolist() for n in (37, 5, 70)]
    pool = S.PagePool(dm, 40)
    opool = np.zeros(40 * om.page_elements, dtype=np.float32)
    caches = [dm.new_cache(pool) for _ in prompts]
    cursor = [0, 0, 0]
    plan = [[16, 5, 33], [16, 1, 37], [5, 1, 1], [1, 1, 1], [1, 1, 1]]
    last = [None] * 3
    for counts in plan:
        chunks, want = [], []
        for i, k in enumerate(counts):
            if cursor[i] < len(prompts[i]):
                chunks.append(prompts[i][cursor[i]:cursor[i] + k])
            else:
                chunks.append([last[i]])
            want.append(cursor[i] + len(chunks[-1]) >= len(prompts[i]))
        pos = [c.pos for c in caches]
        got = dm.prefill_selected(caches, chunks, want)
        exp = om.step(opool, pos, chunks, [c.pages for c in caches], want)
        assert_same(got, exp, f"counts {counts}")
        for i in range(3):
            if cursor[i] < len(prompts[i]):
                cursor[i] += len(chunks[i])
            if want[i]:
                last[i] = int(np.argmax(got[i]))
    for c in caches:
        compare_cache_rows(pool, opool, om, c)


def test_smollm_shape_two_layers_q8(oracle, srlib):
    """SmolLM2-135M layer shapes (d=576, 9/3 heads of 64, ff 1536, V 49152) on 2 layers."""
    S = _step_mod()
    om, dm = synthetic_pair(oracle, srlib, "q8", 16, vocab=49152, dim=576, hidden=1536, layers=2, heads=9,
                            kv_heads=3, context=512, tied=True)
    rng = np.random.default_rng(1)
    pool = S.PagePool(dm, 64)
    opool = np.zeros(64 * om.page_elements, dtype=np.float32)
    caches = [dm.new_cache(pool) for _ in range(3)]
    prompts = [rng.integers(0, 49152, size=n).tolist() for n in (40, 17, 64)]
    got = dm.prefill_selected(caches, prompts)
    exp = om.step(opool, [0, 0, 0], prompts, [c.pages for c in caches], threads=8)
    assert_same(got, exp, "smollm prefill")
    toks = [int(np.argmax(g)) for g in got]
    pos = [c.pos for c in caches]
    got = dm.decode_batch(caches, toks)
    exp = om.step(opool, pos, [[t] for t in toks], [c.pages for c in caches], threads=8)
    assert_same(got, exp, "smollm decode")


def test_mistral_shape_one_layer_q8(oracle, srlib):
    """Mistral-7B layer shapes (d=4096, 32/8 heads of 128, ff 14336) on one layer."""
    S = _step_mod()
    om, dm = synthetic_pair(oracle, srlib, "q8", 16, vocab=2048, dim=4096, hidden=14336, layers=1, heads=32,
                            kv_heads=8, context=256, tied=False)
    rng = np.random.default_rng(2)
    pool = S.PagePool(dm, 16)
    opool = np.zeros(16 * om.page_elements, dtype=np.float32)
    caches = [dm.new_cache(pool) for _ in range(2)]
    prompts = [rng.integers(0, 2048, size=n).tolist() for n in (21, 9)]
    got = dm.prefill_selected(caches, prompts)
    exp = om.step(opool, [0, 0], prompts, [c.pages for c in caches], threads=8)
    assert_same(got, exp, "mistral prefill")
    toks = [int(np.argmax(g)) for g in got]
    got = dm.decode_batch(caches, toks)
    exp = om.step(opool, [21, 9], [[t] for t in toks], [c.pages for c in caches], threads=8)
    assert_same(got, exp, "mistral decode")


def test_wide_rows_take_fp64_path(oracle, srlib):
    """A huge norm weight drives linear inputs above the wide limit (M:4346-4382)."""
    om, dm = synthetic_pair(oracle, srlib, "q8", 32)
    d = om.cfg.dim
    big = np.full(d, 1e35, dtype=np.float32)
    om.set_param_raw(1, big, None)
    dm.load_param(1, big)
    S = _step_mod()
    pool = S.PagePool(dm, 4)
    opool = np.zeros(4 * om.page_elements, dtype=np.float32)
    cache = dm.new_cache(pool)
    got = dm.prefill_selected([cache], [[1, 2, 3]])
    exp = om.step(opool, [0], [[1, 2, 3]], [cache.pages])
    assert_same(got, exp, "wide rows")


def test_invalid_batches_mutate_nothing(oracle, srlib):
    """prefill_test.go:91: invalid input leaves earlier KV untouched."""
    from sr_go_tranformer_b200 import _abi as A
    om, dm = synthetic_pair(oracle, srlib, "q8", 16)
    S = _step_mod()
    pool = S.PagePool(dm, 8)
    cache = dm.new_cache(pool)
    dm.prefill_selected([cache], [[1, 2, 3, 4, 5]])
    snap = [pool.read_row(p, l, s) for p in cache.pages for l in range(2) for s in range(16)]

    def raw_step(pos, toff, tokens, poff, pids, want=None):
        arrs = [np.asarray(x, dtype=np.int32) for x in (pos, toff, tokens, poff, pids)]
        b = A.Batch(len(pos), *[a.ctypes.data for a in arrs], None)
        return A.lib().sr_step(dm.h, pool.h, C.byref(b), None, None)

    V = om.cfg.vocab
    cases = [
        ([5], [0, 1], [V], [0, 1], cache.pages),               # token outside vocabulary
        ([5], [0, 0], [1], [0, 1], cache.pages),               # empty chunk
        ([5], [0, 1], [1], [0, 0], []),                        # no page coverage
        ([300], [0, 1], [1], [0, 1], cache.pages),             # position past context
        ([5], [0, 1], [1], [0, 1], [99]),                      # page id outside the pool
        ([5, 0], [0, 1, 2], [1, 1], [0, 1, 2], cache.pages * 2),  # written page shared by two sessions
        ([-1], [0, 1], [1], [0, 1], cache.pages),              # negative position
    ]
    for pos, toff, tokens, poff, pids in cases:
        assert raw_step(pos, toff, tokens, poff, pids) == A.SR_EINVAL, (pos, toff, tokens)
    after = [pool.read_row(p, l, s) for p in cache.pages for l in range(2) for s in range(16)]
    for (k0, v0), (k1, v1) in zip(snap, after):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
    with pytest.raises(A.SRError):
        dm.prefill_selected([cache], [list(range(1025))])
    assert cache.pos == 5


def test_cancel_flag_commits_nothing(oracle, srlib):
    from sr_go_tranformer_b200 import _abi as A
    om, dm = synthetic_pair(oracle, srlib, "q8", 16)
    S = _step_mod()
    pool = S.PagePool(dm, 8)
    cache = dm.new_cache(pool)
    flag = C.c_int32(1)
    with pytest.raises(A.SRError) as e:
        dm.prefill_selected([cache], [[1, 2, 3]], cancel=flag)
    assert e.value.code == A.SR_ECANCELED
    assert cache.pos == 0
    flag.value = 0
    dm.prefill_selected([cache], [[1, 2, 3]], cancel=flag)  # retry after cancellation is correct
    assert cache.pos == 3


def test_device_synthetic_init_matches_oracle(oracle, srlib):
    """Counter-based device generator == sequential SplitMix64 generator.
    CUDA's and glibc's fp64 log/cos may differ in the last ulp, which can move
    a rare value by one float32 ulp and so a rare Q8 code by one step."""
    cfg = oracle.make_config(300, 64, 96, 2, 4, 2, 128, weight_format="q8")
    om = oracle.Model(cfg)
    om.init_synthetic(77)
    S = _step_mod()
    dm = S.Model(S.make_desc(300, 64, 96, 2, 4, 2, 128, weight_format="q8"))
    dm.init_synthetic(77)
    total = mism = 0
    for i in range(om.nparams):
        a, sa = om.get_param_raw(i)
        b, sb = dm.read_param(i)
        total += a.size
        mism += int(np.sum(a != b))
        if sa is not None:
            assert np.allclose(sa, sb, rtol=1e-6, atol=0)
    assert mism <= max(2, total // 100000), (mism, total)


SETTINGS = [(0.0, 0, 1.0, 1.0), (0.0, 40, 0.95, 1.1), (0.8, 40, 0.95, 1.1), (1.0, 1, 1.0, 1.0), (1.3, 256, 0.5, 2.0),
            (0.8, 7, 1.0, 1.0)]


@pytest.mark.parametrize("vocab", [300, 49152])
def test_sampler_matches_oracle(oracle, srlib, vocab):
    om, dm = synthetic_pair(oracle, srlib, "q8", 16, vocab=vocab)
    S = _step_mod()
    pool = S.PagePool(dm, 64)
    rng = np.random.default_rng(vocab)
    n = len(SETTINGS)
    caches = [dm.new_cache(pool) for _ in range(n)]
    prompts = [rng.integers(0, vocab, size=int(rng.integers(2, 20))).tolist() for _ in range(n)]
    logits = dm.prefill_selected(caches, prompts)
    states = [int(s) for s in rng.integers(0, 2**63, size=n)]
    hist = [p + rng.integers(0, vocab, size=3).tolist() for p in prompts]
    for blocked in (-1, 3):
        ids, new_states = dm.sample(SETTINGS, hist, states, blocked=blocked)
        for i, (t, k, p, pen) in enumerate(SETTINGS):
            want, st = oracle.sample(logits[i], hist[i], t, k, p, pen, states[i], blocked)
            assert ids[i] == want and int(new_states[i]) == st, (i, SETTINGS[i], ids[i], want)


def test_engine_matches_oracle_simulation(oracle, srlib):
    """Scheduling, page tables and every output token are bit-exact with the
    oracle restatement of Engine.run (scheduler_test.go, monolith_test.go:937)."""
    from engine_sim import simulate
    from sr_go_tranformer_b200.engine import Engine
    om, dm = synthetic_pair(oracle, srlib, "q8", 16, vocab=300)
    rng = np.random.default_rng(9)
    reqs = []
    for i in range(7):
        r = dict(ids=rng.integers(0, 300, size=int(rng.integers(1, 40))).tolist(), max_tokens=int(rng.integers(1, 12)),
                 seed=100 + i)
        if i % 2:
            r.update(temperature=0.8, top_k=40, top_p=0.95, penalty=1.1)
        reqs.append(r)
    limit = 24
    page_bytes = om.page_elements * 4
    eng = Engine(dm, max_batch=4, token_budget=16, prefill_chunk=8, mixed_prefill_chunk=2,
                 cache_bytes=limit * page_bytes, eos_id=299)
    for r in reqs:
        eng.submit(r["ids"], r["max_tokens"], r.get("temperature", 0.0), r.get("top_k", 0), r.get("top_p", 1.0),
                   r.get("penalty", 1.0), r["seed"])
    done = eng.run_to_completion()
    want, trace = simulate(om, reqs, limit, 4, 16, 8, 2, eos_id=299)
    assert set(done) == set(want)
    for k in want:
        assert done[k][0] == want[k][0], (k, done[k], want[k])
        assert done[k][1] == want[k][1]
    st = eng.stats()
    assert st["active"] == 0 and st["pool_reserved"] == 0
    # firstTokenLatency / tokenGap observations (M:8441-8447): one first token per
    # request that produced any token, one gap for every later token
    lat = eng.latency()
    produced = [k for k in want if len(want[k][0]) > 0]
    assert lat["first_tokens"] == len(produced)
    assert lat["gaps"] == st["generated_tokens"] - len(produced)
    assert lat["ttft_p50_ms"] > 0 and lat["itl_p50_ms"] > 0


def test_kvpool_copy_rows(oracle, srlib):
    """sr_kvpool_copy_rows restates copyKVPrefixRows (M:5907-5914): the first
    `rows` slots of every layer's K and V planes move bit for bit, the rest of
    the destination page is untouched."""
    S = _step_mod()
    om, dm = synthetic_pair(oracle, srlib, "q8", 16)
    pool = S.PagePool(dm, 8)
    pool.fill_synthetic(5, 1.0)
    pt, L = om.cfg.page_tokens, om.cfg.layers
    before = {(p, l, s): pool.read_row(p, l, s) for p in (2, 6) for l in range(L) for s in range(pt)}
    pool.copy_rows(6, 2, 5)
    for l in range(L):
        for s in range(pt):
            k, v = pool.read_row(6, l, s)
            src = before[(2, l, s)] if s < 5 else before[(6, l, s)]
            assert_same(k, src[0], f"K layer {l} slot {s}")
            assert_same(v, src[1], f"V layer {l} slot {s}")
    pool.copy_rows(6, 2, pt)  # whole page
    for l in range(L):
        for s in range(pt):
            k, v = pool.read_row(6, l, s)
            assert_same(k, before[(2, l, s)][0], "K full")
            assert_same(v, before[(2, l, s)][1], "V full")
    for bad in ((8, 2, 1), (6, -1, 1), (6, 2, pt + 1), (6, 2, -1)):
        with pytest.raises(Exception):
            pool.copy_rows(*bad)


def _prefix_requests(seed, n, system=40, vocab=300):
    rng = np.random.default_rng(seed)
    head = rng.integers(0, vocab, size=system).tolist()
    reqs = []
    for i in range(n):
        r = dict(ids=head + rng.integers(0, vocab, size=int(rng.integers(1, 9))).tolist(),
                 max_tokens=int(rng.integers(2, 6)), seed=70 + i)
        if i % 2:
            r.update(temperature=0.7, top_k=20, top_p=0.9, penalty=1.1)
        reqs.append(r)
    return reqs


def _run_engine(eng, reqs):
    ids = [eng.submit(r["ids"], r["max_tokens"], r.get("temperature", 0.0), r.get("top_k", 0), r.get("top_p", 1.0),
                      r.get("penalty", 1.0), r["seed"]) for r in reqs]
    done = eng.run_to_completion()
    return {i: done[rid] for i, rid in enumerate(ids)}


@pytest.mark.parametrize("tail,max_batch", [(False, 1), (True, 1), (True, 3)])
def test_engine_prefix_cache_matches_simulation(oracle, srlib, tail, max_batch):
    """The C++ engine's prefix snapshot (restore M:5881-5905 at admission,
    capture M:5927-5952 at finish, device page copies) against the oracle
    simulation: identical outputs, hits and reused tokens, and the outputs of
    an engine without the cache."""
    from engine_sim import simulate
    from sr_go_tranformer_b200.engine import Engine
    om, dm = synthetic_pair(oracle, srlib, "q8", 16, vocab=300)
    reqs = _prefix_requests(12, 6)
    limit, plimit = 24, 4
    page_bytes = om.page_elements * 4
    eng = Engine(dm, max_batch=max_batch, token_budget=16, prefill_chunk=8, mixed_prefill_chunk=1,
                 cache_bytes=(limit + plimit) * page_bytes, prefix_cache_bytes=plimit * page_bytes,
                 prefix_cache_tail=tail)
    got = _run_engine(eng, reqs)
    st = eng.stats()
    sim = {}
    want, _ = simulate(om, reqs, limit, max_batch, 16, 8, 1, prefix_limit=plimit, prefix_tail=tail, stats=sim)
    base, _ = simulate(om, reqs, limit, max_batch, 16, 8, 1)
    assert want == base
    for k in want:
        assert got[k] == want[k], (k, got[k], want[k])
    assert st["prefix_hits"] == sim["prefix_hits"] > 0
    assert st["prefix_tokens"] == sim["prefix_tokens"]
    assert st["prefix_bytes"] == sim["prefix_pages"] * page_bytes
    assert st["pool_limit"] == limit and st["pool_reserved"] == 0 and st["active"] == 0
    # clearPrefix (M:8236-8241): applied at once when idle; the next request
    # finds no snapshot
    eng.clear_prefix()
    assert eng.stats()["prefix_bytes"] == 0
    again = _run_engine(eng, reqs[1:2])
    assert again[0] == want[1]
    assert eng.stats()["prefix_hits"] == st["prefix_hits"]
    eng.close()


def test_engine_prefix_config_errors(oracle, srlib):
    """normalizeEngineConfig / newEngine prefix checks (M:7999-8003, 8031-8034)."""
    from sr_go_tranformer_b200.engine import Engine
    om, dm = synthetic_pair(oracle, srlib, "q8", 16, vocab=300)
    pb = om.page_elements * 4
    for kw in (dict(cache_bytes=8 * pb, prefix_cache_bytes=8 * pb), dict(cache_bytes=8 * pb, prefix_cache_bytes=-1),
               dict(cache_bytes=8 * pb, prefix_cache_tail=True), dict(cache_bytes=8 * pb, prefix_cache_bytes=pb // 2)):
        with pytest.raises(Exception):
            Engine(dm, max_batch=2, **kw)
    e = Engine(dm, max_batch=2, cache_bytes=8 * pb, prefix_cache_bytes=3 * pb)
    assert e.stats()["pool_limit"] == 5
    e.close()


@pytest.mark.parametrize("table", ["hf-bytes", "mistral-fallback"])
def test_engine_token_events(oracle, srlib, table):
    """TokenEvent (M:8451-8462): one event per sampled token, in order, whose
    texts concatenate to the decoder's text of the request's pieces; the last
    is final.  "hf-bytes": byte-level pieces where some ids hold half of a
    multi-byte character.  "mistral-fallback": a SentencePiece-style table where
    a third of the ids are byte-fallback tokens holding single bytes of
    multi-byte characters (runs may end a request part-way: the final event
    flushes them) and the rest are pieces with the leading-space marker."""
    from sr_go_tranformer_b200.engine import Engine
    from sr_go_tranformer_b200.text import TextDecoder
    om, dm = synthetic_pair(oracle, srlib, "q8", 16, vocab=300)
    if table == "hf-bytes":
        euro = "€".encode()
        pieces = [bytes([97 + i % 26]) if i % 7 else euro[:2] if i % 2 else euro[2:] for i in range(300)]
        flags, fallback = dict(hf=True), None
    else:
        utf8 = "€ü世".encode()  # 3 + 2 + 3 bytes
        fallback = np.array([1 if i % 3 == 0 else 0 for i in range(300)], dtype=np.uint8)
        pieces = [bytes([utf8[(i // 3) % len(utf8)]]) if fallback[i] else ("\u2581" * (i % 2) + chr(97 + i % 26)).encode()
                  for i in range(300)]
        flags = dict(mistral=True, fallback=fallback)
    eng = Engine(dm, max_batch=2, token_budget=16, prefill_chunk=8, mixed_prefill_chunk=1,
                 cache_bytes=24 * om.page_elements * 4)
    eng.set_pieces(pieces, **flags)
    rng = np.random.default_rng(3)
    rids = [eng.submit(rng.integers(0, 300, size=int(rng.integers(2, 20))).tolist(), int(rng.integers(2, 9)),
                       0.9, 20, 0.9, 1.0, 11 + i) for i in range(3)]
    done = eng.run_to_completion()
    events = {}
    while True:
        ev = eng.poll_token()
        if ev is None:
            break
        events.setdefault(ev[0], []).append(ev[1:])
    for rid in rids:
        out, _ = done[rid]
        evs = events[rid]
        assert [t for t, _, _ in evs] == out
        assert [f for _, _, f in evs] == [False] * (len(out) - 1) + [True]
        d = TextDecoder(**flags)
        want = "".join(d.push_token(t, pieces[t], k == len(out) - 1) for k, t in enumerate(out))
        assert "".join(x for _, x, _ in evs) == want
    eng.close()
