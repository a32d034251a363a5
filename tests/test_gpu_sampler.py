"""GPU parity of the device sampler (sampleWithBlocked, M:7320-7426, with the
SplitMix64 RNG, M:1411-1439) against the oracle's full-sort restatement, on the
reference's own sampler grids.

Every case samples through the C ABI (`sr_sample_logits`, the device path of
`sr_sample`) and must give the oracle's token id and RNG state bit for bit;
error cases must fail with SR_EINVAL and leave the RNG state untouched.  The
inputs are generated as the reference's tests generate them (the same
SplitMix64 draws), so the grids are the reference's:
  - topk_sampling_test.go:60-112  (TestBoundedTopKSamplingExact): sizes
    8/33/258/1024 with signed zeros, every k edge (0, 1, size/4, size/4+1,
    size-1, size, size+1), blocked -1 / size/2, temperatures .01/.8/100, top-p
    .01/.95/1, penalties 1/1.1, seeds 1/42/MaxUint64; vocabularies 32768 and
    151936 at the default settings;
  - topk_sampling_test.go:114-133 (discarded nonfinite values, all-zero and
    extreme logits);
  - sampling_test.go:96-128 (greedy fixtures: ties, signed zero, subnormals,
    MaxFloat32, penalties 1/1.1/2/100, blocked -1/0/len/2/len);
  - sampling_test.go:129-149 (empty and nonfinite distributions);
  - sampling_test.go:151-166 (sampled path: temperatures .01/.8/2/100, top-k
    0/1/40/1000, top-p .01/.7/1, blocked -1/0/258).
top_k 0 and top_k above 256 take the device's full-vocabulary sort
(k_sample_full); the others the bounded radix select (k_sample).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32_MAX = float(np.finfo(np.float32).max)
F32_TINY = float(np.float32(1.4e-45))  # math.SmallestNonzeroFloat32
U64_MAX = 2**64 - 1
DEFAULT = (0.8, 40, 0.95, 1.1)  # defaultSampling (M:7262)


@pytest.fixture(scope="module")
def dm(srlib):
    from sr_go_tranformer_b200 import step as S
    m = S.Model(S.make_desc(300, 64, 64, 1, 2, 1, 64))
    yield m
    m.close()


def _oracle(oracle, logits, hist, setting, seed, blocked):
    t, k, p, pen = setting
    try:
        return oracle.sample(logits, hist, t, k, p, pen, seed, blocked)
    except ValueError:
        return None


def _raw_sample(dm, logits, settings, hists, seeds, blocked):
    """sr_sample_logits through ctypes; returns (rc, ids, rng states after the call)."""
    import ctypes as C
    from sr_go_tranformer_b200 import _abi as A
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    n = lg.shape[0]
    arr = (A.Sampling * n)(*[A.Sampling(t, k, 0, p, pen) for t, k, p, pen in settings])
    hoff = np.zeros(n + 1, dtype=np.int32)
    hoff[1:] = np.cumsum([len(h) for h in hists])
    hist = np.concatenate([np.asarray(h, dtype=np.int32) for h in hists] + [np.zeros(1, np.int32)])
    rng = np.asarray(seeds, dtype=np.uint64).copy()
    ids = np.full(n, -1, dtype=np.int32)
    rc = A.lib().sr_sample_logits(dm.h, n, lg.shape[1], lg.ctypes.data, C.cast(arr, C.c_void_p), hoff.ctypes.data,
                                  hist.ctypes.data, rng.ctypes.data, blocked, ids.ctypes.data)
    return rc, ids, rng


def run_cases(oracle, dm, logits, hist, cases, blocked):
    """cases: list of (setting, seed) on one logits row; device calls of up to
    256 sessions; error cases go one by one and must fail with SR_EINVAL
    leaving the caller's RNG state as it was.  Returns the number compared."""
    from sr_go_tranformer_b200 import _abi as A
    want = [_oracle(oracle, logits, hist, s, seed, blocked) for s, seed in cases]
    ok = [i for i, w in enumerate(want) if w is not None]
    for c0 in range(0, len(ok), 256):
        idx = ok[c0:c0 + 256]
        lg = np.tile(np.asarray(logits, dtype=np.float32), (len(idx), 1))
        ids, st = dm.sample_logits(lg, [cases[i][0] for i in idx], [hist] * len(idx),
                                   [cases[i][1] for i in idx], blocked)
        for j, i in enumerate(idx):
            assert (int(ids[j]), int(st[j])) == want[i], (cases[i], blocked, int(ids[j]), want[i])
    for i, w in enumerate(want):
        if w is not None:
            continue
        rc, _, st = _raw_sample(dm, np.asarray(logits, dtype=np.float32)[None, :], [cases[i][0]], [hist],
                                [cases[i][1]], blocked)
        assert rc == A.SR_EINVAL and int(st[0]) == cases[i][1] % 2**64, (cases[i], blocked, rc)
    return len(cases)


def topk_inputs(oracle):
    """The logits of TestBoundedTopKSamplingExact, drawn from one RNG{19}
    stream in the test's order (sizes 8, 33, 258, 1024, then 32768, 151936)."""
    rnd = oracle.RNG(19)
    out = {}
    for size in (8, 33, 258, 1024):
        x = np.zeros(size, dtype=np.float32)
        for i in range(size):
            x[i] = np.float32(rnd.intn(65) - 32) / np.float32(7)
            if i % 7 == 0:
                x[i] = np.float32(-0.0)
        out[size] = x
    for size in (32768, 151936):
        out[size] = np.array([np.float32(rnd.intn(10000) - 5000) / np.float32(19) for _ in range(size)],
                             dtype=np.float32)
    return out


@pytest.fixture(scope="module")
def topk(oracle):
    return topk_inputs(oracle)


def test_bounded_topk_grid(oracle, dm, topk):
    """TestBoundedTopKSamplingExact (topk_sampling_test.go:60-95)."""
    n = 0
    for size in (8, 33, 258, 1024):
        logits = topk[size]
        hist = [0, 1, 1, size // 2, size - 1, -1, size + 1]
        for blocked in (-1, size // 2):
            cases = [((t, k, p, pen), seed)
                     for k in (0, 1, size // 4, size // 4 + 1, size - 1, size, size + 1)
                     for t in (.01, .8, 100) for p in (.01, .95, 1) for pen in (1, 1.1) for seed in (1, 42, U64_MAX)]
            n += run_cases(oracle, dm, logits, hist, cases, blocked)
    assert n == 4 * 2 * 7 * 3 * 3 * 2 * 3


@pytest.mark.parametrize("size", [32768, 151936])
def test_large_vocabulary(oracle, dm, topk, size):
    """topk_sampling_test.go:96-111 (default settings, seeds 19/42), plus the
    full-vocabulary path at the same sizes (top_k 0 and 1000)."""
    logits = topk[size]
    cases = [(DEFAULT, 19), (DEFAULT, 42), ((0.8, 0, 0.95, 1.1), 19), ((0.8, 0, 1.0, 1.0), 42),
             ((2.0, 1000, 0.7, 1.1), 42), ((100.0, 0, 1.0, 1.1), 7), ((0.0, 0, 1.0, 1.1), 1)]
    run_cases(oracle, dm, logits, [0, 40, 40], cases, -1)
    run_cases(oracle, dm, logits, [0, 40, 40], cases, size // 3)


def test_discarded_nonfinite_and_extremes(oracle, dm):
    """TestBoundedTopKRejectsDiscardedNonfinite (topk_sampling_test.go:114-133)."""
    for bad in (np.nan, np.inf, -np.inf):
        for blocked in (-1, 127):
            logits = np.zeros(128, dtype=np.float32)
            logits[0] = F32_MAX
            logits[127] = bad
            for k in (1, 0, 300):
                run_cases(oracle, dm, logits, [], [((0.8, k, 0.95, 1.1), 19)], blocked)
    for logits in ([0.0] * 8, [F32_MAX, -F32_MAX, F32_TINY, 0, 0, 0, 0, 0]):
        for k in (1, 2, 0):
            run_cases(oracle, dm, np.asarray(logits, dtype=np.float32), [0, 0, 1],
                      [((0.8, k, 0.95, 1.1), 42), ((0.0, k, 0.95, 1.1), 42)], -1)


def test_greedy_fixtures(oracle, dm):
    """TestGreedyMatchesSortedReference (sampling_test.go:96-128)."""
    fixtures = [[0], [3, 3, 3], [-3, -3, -3], [-10, -2, -4], [-0.0, 0, -1], [F32_TINY, 0, -F32_TINY],
                [F32_MAX, -F32_MAX, F32_MAX], [20, 10, 5]]
    rnd = oracle.RNG(17)
    for _ in range(128):
        size = 1 + rnd.intn(1024)
        fixtures.append([np.float32(rnd.intn(101) - 50) / np.float32(7) for _ in range(size)])
    for f in fixtures:
        logits = np.asarray(f, dtype=np.float32)
        hist = [0, 0, 1, 3, -1, len(f) + 1]
        for blocked in (-1, 0, len(f) // 2, len(f)):
            cases = [((0.0, 40, 0.95, pen), 42) for pen in (1, 1.1, 2, 100)]
            run_cases(oracle, dm, logits, hist, cases, blocked)


def test_invalid_distributions(oracle, dm):
    """TestSamplingInvalidDistributions (sampling_test.go:129-149): an empty
    distribution and nonfinite logits (also masked ones) are errors that leave
    the RNG state unchanged."""
    from sr_go_tranformer_b200 import _abi as A
    for t in (0.0, 0.8):
        for k in (40, 0):
            rc, _, st = _raw_sample(dm, np.ones((1, 1), np.float32), [(t, k, 0.95, 1.1)], [[]], [1], 0)
            assert rc == A.SR_EINVAL and int(st[0]) == 1
        for bad in (np.nan, np.inf, -np.inf):
            for row in ([bad, 1], [1, bad], [100, 0, bad]):
                for blocked in (-1, 0, len(row) - 1):
                    for k in (40, 0):
                        rc, _, st = _raw_sample(dm, np.asarray([row], np.float32), [(t, k, 0.95, 1.1)], [[]],
                                                [12345], blocked)
                        assert rc == A.SR_EINVAL and int(st[0]) == 12345


def test_sampled_path(oracle, dm):
    """TestSampledPathMatchesSortedReference (sampling_test.go:151-166)."""
    rnd = oracle.RNG(37)
    logits = np.array([np.float32(rnd.intn(1000) - 500) / np.float32(13) for _ in range(259)], dtype=np.float32)
    for blocked in (-1, 0, 258):
        cases = [((t, k, p, 1.1), 42) for t in (.01, .8, 2, 100) for k in (0, 1, 40, 1000) for p in (.01, .7, 1)]
        run_cases(oracle, dm, logits, [0, 7, 128, 128], cases, blocked)


def test_full_path_ragged_sessions(oracle, dm):
    """Many sessions in one call, each with its own logits, history and settings,
    more than one wave of the full-vocabulary kernel (32 sessions per launch),
    mixed with bounded and greedy sessions."""
    rng = np.random.default_rng(3)
    n, V = 80, 5000
    logits = (rng.standard_normal((n, V)) * 3).astype(np.float32)
    logits[:, ::11] = np.round(logits[:, ::11])  # ties
    settings = [((0.7, [0, 257, 4999, 5000, 40, 0][i % 6], [1.0, 0.9, 0.3][i % 3], [1.0, 1.3][i % 2]))
                if i % 5 else (0.0, 0, 1.0, 1.2) for i in range(n)]
    hists = [rng.integers(0, V, size=int(rng.integers(0, 50))).tolist() for _ in range(n)]
    seeds = [int(s) for s in rng.integers(0, 2**63, size=n)]
    ids, st = dm.sample_logits(logits, settings, hists, seeds, 17)
    for i in range(n):
        t, k, p, pen = settings[i]
        assert (int(ids[i]), int(st[i])) == oracle.sample(logits[i], hists[i], t, k, p, pen, seeds[i], 17), i
