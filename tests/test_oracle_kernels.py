"""Oracle kernel, quantizer, sampler, RNG and scheduler checks (CPU).

Ports the reference's own known-answer and property tests for the hot path:
  q8_test.go:38 (scale extremes), q8_test.go:55 (Q8 linear vs fp64 dot of the
  reconstructed weights, rel 2e-5), q8_test.go:194-291 (quantized model ==
  dense model over reconstructed weights within 3e-5), monolith_test.go:1076
  (sampler bounds and determinism), scheduler_test.go:18 (token budget).
"""

import numpy as np
import pytest

from conftest import GOLDEN


def test_splitmix64_known_answers(oracle):
    # Published SplitMix64 outputs for seed 1234567 (Vigna's reference code).
    r = oracle.RNG(1234567)
    got = [r.uint64() for _ in range(5)]
    assert got == [6457827717110365317, 3203168211198807973, 9817491932198370423, 4593380528125082431,
                   16408922859458223821]


def test_rng_float_and_intn(oracle):
    r = oracle.RNG(7)
    for _ in range(1000):
        f = r.float64()
        assert 0.0 <= f < 1.0
    r = oracle.RNG(9)
    vals = [r.intn(258) for _ in range(2000)]
    assert min(vals) >= 0 and max(vals) < 258 and len(set(vals)) > 200


def test_q8_scale_extremes(oracle):
    L = oracle.lib()
    fmax = float(np.finfo(np.float32).max)
    tiny = float(np.finfo(np.float32).smallest_subnormal)
    for amax in [0.0, tiny, 1e-43, 1e-37, 0.03, 1.0, fmax]:
        amax = float(np.float32(amax))
        s = L.or_low_bit_scale(amax, 127.0)
        assert np.isfinite(s) and s >= 0 and (amax == 0 or s > 0)
        for x in [-amax, -amax / 3, 0.0, amax / 3, amax]:
            x = float(np.float32(x))
            q = L.or_q8_value(x, s)
            got = float(np.float32(q) * np.float32(s))
            assert np.isfinite(got) and q >= -127
            assert abs(got - x) <= s * 0.501 + amax * 2e-7


@pytest.mark.parametrize("fmt", [1, 2])
@pytest.mark.parametrize("inp", [1, 2, 63, 64, 65, 129, 513])
def test_quantized_linear_vs_fp64(oracle, fmt, inp):
    rng = np.random.default_rng(inp * 10 + fmt)
    out, n = 37, 5
    w = rng.uniform(-1, 1, (out, inp)).astype(np.float32)
    x = rng.uniform(-1, 1, (n, inp)).astype(np.float32)
    vals, scales = oracle.quantize(w, fmt)
    groups = (inp + 63) // 64
    recon = np.zeros((out, inp), dtype=np.float64)
    for o in range(out):
        row = np.zeros(inp, dtype=np.float32)
        oracle.lib().or_copy_row(vals.ctypes.data, scales.ctypes.data, fmt, inp, o, row.ctypes.data)
        recon[o] = row
    y = oracle.linear(x, fmt, vals, scales, out, inp)
    ref = x.astype(np.float64) @ recon.T
    scale = np.abs(x.astype(np.float64)) @ np.abs(recon).T + 1e-30
    assert np.max(np.abs(y - ref) / scale) <= 2e-5
    # batch determinism: each row alone gives the same bits
    for r in range(n):
        y1 = oracle.linear(x[r:r + 1], fmt, vals, scales, out, inp)
        assert np.array_equal(y1[0], y[r])
    # thread-count invariance
    y4 = oracle.linear(x, fmt, vals, scales, out, inp, threads=4)
    assert np.array_equal(y4, y)
    assert groups >= 1


def test_wide_rows_select_per_row(oracle):
    """An extreme row takes the fp64 path without changing its neighbours (M:4359-4365)."""
    rng = np.random.default_rng(3)
    out, inp = 9, 130
    w = rng.uniform(-1, 1, (out, inp)).astype(np.float32)
    vals, scales = oracle.quantize(w, 1)
    x = rng.uniform(-1, 1, (3, inp)).astype(np.float32)
    base = oracle.linear(x, 1, vals, scales, out, inp)
    x2 = x.copy()
    x2[1, 5] = 3e34  # above float32(MaxFloat32/(2*64*127))
    y = oracle.linear(x2, 1, vals, scales, out, inp)
    assert np.array_equal(y[0], base[0]) and np.array_equal(y[2], base[2])
    assert np.all(np.isfinite(y[1]))


@pytest.mark.parametrize("fmt", ["q8", "q4", "q4-mixed"])
def test_quantized_model_matches_reconstructed_dense(oracle, fmt):
    """q8_test.go:194-291: a quantized model equals a dense model built from the
    reconstructed weights within 3e-5, across chunks 33,1,7,1."""
    mq, z, hf = oracle.load_golden(GOLDEN[0], weight_format=fmt)
    md = oracle.Model(oracle.config_from_hf(hf))
    for i in range(mq.nparams):
        info = mq.param_info(i)
        vals, sc = mq.get_param_raw(i)
        if info.format == 0:
            md.set_param_raw(i, vals, None)
            continue
        recon = np.zeros((info.rows, info.cols), dtype=np.float32)
        for r in range(info.rows):
            oracle.lib().or_copy_row(vals.ctypes.data, sc.ctypes.data, info.format, info.cols, r,
                                     recon[r].ctypes.data)
        md.set_param_raw(i, recon, None)
    ids = z["ids"]
    pq = np.zeros(2 * mq.page_elements, dtype=np.float32)
    pd = np.zeros(2 * md.page_elements, dtype=np.float32)
    pos = 0
    for chunk in (33, 1, 2, 1):
        a = mq.step(pq, [pos], [ids[pos:pos + chunk]], [[0, 1]])
        b = md.step(pd, [pos], [ids[pos:pos + chunk]], [[0, 1]])
        assert np.abs(a - b).max() <= 3e-5
        pos += chunk


def test_quantizer_odd_widths_q4(oracle):
    rng = np.random.default_rng(11)
    w = rng.uniform(-2, 2, (3, 65)).astype(np.float32)
    vals, sc = oracle.quantize(w, 2)
    assert vals.size == 3 * 33 and sc.size == 3 * 2
    # high pad nibble of odd rows stays zero (q4Weights, M:3804-3809)
    assert all((vals[r * 33 + 32] >> 4) == 0 for r in range(3))


def test_sampler_bounds_and_determinism(oracle):
    """monolith_test.go:1076-1106 (BOS=256 blocked for native vocab)."""
    logits = np.zeros(258, dtype=np.float32)
    logits[256], logits[17], logits[18] = 100, 10, 9
    s = oracle.sample
    assert s(logits, [], 0.0, 40, 0.95, 1.1, 1, blocked=256)[0] == 17
    assert s(logits, [17], 0.0, 40, 0.95, 2.0, 1, blocked=256)[0] == 18
    for i in range(50):
        assert s(logits, [], 1.0, 1, 0.95, 2.0, i, blocked=256)[0] == 17
    assert s(logits, [], 1.0, 0, 0.01, 2.0, 42, blocked=256)[0] == 17


def test_sampler_greedy_consumes_no_rng(oracle):
    logits = np.array([0.0, -0.0, 3.0, 3.0], dtype=np.float32)
    idx, st = oracle.sample(logits, [], 0.0, 0, 1.0, 1.0, 42)
    assert idx == 2 and st == 42


def test_sampler_nonfinite_and_empty(oracle):
    with pytest.raises(ValueError):
        oracle.sample(np.array([0, np.inf], dtype=np.float32), [], 0.0, 0, 1.0, 1.0, 1)
    with pytest.raises(ValueError):
        oracle.sample(np.array([1.0], dtype=np.float32), [], 0.0, 0, 1.0, 1.0, 1, blocked=0)


def test_scheduler_budget_and_decode_progress(oracle):
    """scheduler_test.go:18-57."""
    ids_len = [2, 3, 100, 100]
    cursor = [2, 2, 0, 0]
    rem = [ids_len[i] - cursor[i] for i in range(4)]
    extra = [0] * 4
    for tick in range(12):
        counts, total = oracle.schedule_tokens(rem, 5, 4, 4, tick % 4)
        assert total == 5
        assert all(1 <= c <= 4 for c in counts)
        assert counts[0] == 1 and counts[1] == 1 and sum(counts) == total
        for i in range(4):
            extra[i] += counts[i] - 1
    assert extra[2] > 0 and extra[3] > 0
    counts, total = oracle.schedule_tokens(rem, 1024, 16, 16, 0)
    assert total == 34 and counts[2] == 16 and counts[3] == 16
    counts, total = oracle.schedule_tokens(rem, 64, 16, 1, 0)
    assert total == 4
    rem[0] = 2
    counts, total = oracle.schedule_tokens(rem, 64, 16, 1, 0)
    assert total > 4


def test_synthetic_init_is_deterministic(oracle):
    cfg = oracle.make_config(258, 32, 48, 2, 4, 2, 64, weight_format="q8")
    a, b = oracle.Model(cfg), oracle.Model(cfg)
    a.init_synthetic(5)
    b.init_synthetic(5)
    for i in range(a.nparams):
        va, sa = a.get_param_raw(i)
        vb, sb = b.get_param_raw(i)
        assert np.array_equal(va, vb)
        if sa is not None:
            assert np.array_equal(sa, sb)


@pytest.mark.parametrize("fmt", ["f32", "q8", "q4"])
def test_parallel_synthetic_init_equals_sequential(oracle, fmt):
    cfg = oracle.make_config(300, 64, 96, 2, 4, 2, 64, weight_format=fmt, qkv_bias=True, tied=False)
    a, b = oracle.Model(cfg), oracle.Model(cfg)
    a.init_synthetic(21)
    b.init_synthetic(21, threads=5)
    for i in range(a.nparams):
        va, sa = a.get_param_raw(i)
        vb, sb = b.get_param_raw(i)
        assert np.array_equal(va, vb)
        if sa is not None:
            assert np.array_equal(sa, sb)
