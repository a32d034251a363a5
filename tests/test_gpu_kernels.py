"""Kernel-level GPU parity through the C ABI: the device quantizer behind
sr_model_load_param_f32 and the exact-order projections behind sr_linear,
bit for bit against the oracle, on the reference's own unit-test grids:

  - the streaming block quantizer (readParam M:857-880, lowBitScale
    M:3877-3891, q8Value M:3893-3898, q4.put M:3819-3822) as the reference's
    quantizeTestParam / quantizeQ4TestParam restate it (q8_test.go:18,
    q4_test.go:69): all-zero blocks, the finite extremes of
    TestQ8ScaleFiniteExtremes (q8_test.go:38: 0, SmallestNonzero, 1e-43,
    1e-37, .03, 1, MaxFloat32), scales that underflow, scales nudged down,
    half-away rounding ties, tails of every length and odd Q4 widths;
  - TestQ8BlocksEveryCodeAndColumn (q8_block_test.go:94): all 256 codes at
    every one of the 64 columns;
  - TestQ4FullBlockEveryCodeAndColumn (q4_block_test.go:11): all 256 packed
    bytes at every column, also against x * value * scale;
  - TestQ8BlocksExactAcrossTailsRowsAndWorkers (q8_block_test.go:127) and
    TestQ4FullBlockAndEveryTailMatchLegacy (q4_block_test.go:40): widths with
    no full block, several blocks and every tail, rows 1..7 (and the larger
    row tiles), subnormal and -0 inputs, zero and subnormal scales;
  - the FP32 sequential dot (linearFP32Range M:3970-4070) on the same widths.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32_MAX = float(np.finfo(np.float32).max)
F32_TINY = np.float32(1.4e-45)
Q8, Q4 = 1, 2
EMB, DOWN = 0, 9  # parameter indices: the embedding [vocab, dim]; layer 0's down_proj [dim, hidden]


def model(vocab=256, dim=64, hidden=64, fmt="q8"):
    from sr_go_tranformer_b200 import step as S
    return S.Model(S.make_desc(vocab, dim, hidden, 1, 1, 1, 64, tied=True, weight_format=fmt))


def bits_equal(a, b, what):
    a = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    b = np.ascontiguousarray(b, dtype=np.float32).view(np.uint32)
    if not np.array_equal(a, b):
        i = np.argwhere(a != b)[0]
        raise AssertionError(f"{what}: {int((a != b).sum())} differ, first at {tuple(i)}: "
                             f"{a.view(np.float32)[tuple(i)]!r} vs {b.view(np.float32)[tuple(i)]!r}")


def special_matrix(rows, cols, levels, seed):
    """Rows of special blocks for the quantizer: zeros, the finite extremes,
    exact half-step ties, tiny and huge magnitudes, then random rows."""
    rng = np.random.default_rng(seed)
    w = np.zeros((rows, cols), dtype=np.float32)
    extremes = [0.0, float(F32_TINY), 1e-43, 1e-37, 0.03, 1.0, F32_MAX]
    r = 0
    for m in extremes:  # TestQ8ScaleFiniteExtremes: {-m, -m/3, 0, m/3, m} repeated
        if r >= rows:
            break
        pat = np.array([-m, -m / 3, 0, m / 3, m], dtype=np.float64).astype(np.float32)
        w[r] = np.resize(pat, cols)
        r += 1
    if r < rows:  # ties: amax = levels gives scale 1; k + 0.5 rounds half away from zero
        ties = np.arange(-levels, levels + 1, dtype=np.float32) + np.float32(0.5)
        ties = np.clip(ties, -levels, levels)
        row = np.resize(np.concatenate([ties, -ties]), cols)
        for g in range(0, cols, 64):
            row[g] = levels  # each block's amax
        w[r] = row
        r += 1
    while r < rows:  # random magnitudes from 1e-44 to 1e37; some blocks all zero, some with one value
        e = rng.uniform(-44, 37)
        row = (rng.standard_normal(cols) * 10.0 ** e).astype(np.float32)
        if r % 7 == 0:
            row[: min(cols, 64)] = 0
        if r % 11 == 0:
            row[:] = 0
            row[rng.integers(0, cols)] = np.float32(10.0 ** e)
        w[r] = row
        r += 1
    return w


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("hidden", [1, 3, 63, 64, 65, 127, 129, 193])
def test_device_quantizer_bit_exact(oracle, srlib, fmt, hidden):
    """sr_model_load_param_f32 quantizes on the device exactly as readParam:
    codes and scales bit for bit (down_proj [64, hidden]: odd Q4 widths and
    every tail length; gate [hidden, 64]: whole blocks)."""
    levels = 127 if fmt == "q8" else 7
    dm = model(hidden=hidden, fmt=fmt)
    for index, (rows, cols) in ((DOWN, (64, hidden)), (7, (hidden, 64)), (EMB, (256, 64))):
        w = special_matrix(rows, cols, levels, seed=hidden * 10 + index)
        dm.load_param_f32(index, w)
        vals, sc = dm.read_param(index)
        wv, ws = oracle.quantize(w, Q8 if fmt == "q8" else Q4)
        assert np.array_equal(vals.view(np.uint8), wv.view(np.uint8)), (fmt, hidden, index)
        bits_equal(sc, ws, f"{fmt} scales hidden {hidden} param {index}")
    dm.close()


def test_q8_every_code_and_column(oracle, srlib):
    """TestQ8BlocksEveryCodeAndColumn: row r of a [256, 64] Q8 matrix holds
    int8(r - 128 + 37 j), scale .25; input rows are the basis vectors 1.25 e_col
    and -0.75 e_(63-col), so every code meets every column in both signs."""
    dm = model(fmt="q8")
    codes = ((np.arange(256)[:, None] - 128 + 37 * np.arange(64)[None, :]) & 255).astype(np.uint8).view(np.int8)
    scales = np.full(256, 0.25, dtype=np.float32)
    dm.load_param(EMB, codes, scales)
    x = np.zeros((128, 64), dtype=np.float32)
    for col in range(64):
        x[2 * col, col] = 1.25
        x[2 * col + 1, 63 - col] = -0.75
    got = dm.linear(EMB, x)
    want = oracle.linear(x, Q8, codes, scales, 256, 64)
    bits_equal(got, want.reshape(got.shape), "q8 every code and column")
    dm.close()


def test_q4_every_code_and_column(oracle, srlib):
    """TestQ4FullBlockEveryCodeAndColumn: row r of a [256, 64] Q4 matrix packs
    bytes (r + 37 j) mod 256, scale .25; x = 1.25 e_col.  Each output equals
    x * value * scale (and the oracle) bit for bit."""
    dm = model(fmt="q4")
    packed = np.array([[(r + 37 * j) & 255 for j in range(32)] for r in range(256)], dtype=np.uint8)
    scales = np.full(256, 0.25, dtype=np.float32)
    dm.load_param(EMB, packed, scales)
    x = np.eye(64, dtype=np.float32) * np.float32(1.25)
    got = dm.linear(EMB, x)
    want = oracle.linear(x, Q4, packed, scales, 256, 64).reshape(got.shape)
    bits_equal(got, want, "q4 every code and column")
    nib = np.zeros((256, 64), dtype=np.int64)
    nib[:, 0::2] = packed & 15
    nib[:, 1::2] = packed >> 4
    val = np.where(nib >= 8, nib - 16, nib).astype(np.float32)
    closed = (np.float32(1.25) * val * np.float32(0.25)).T  # [col, row]
    bits_equal(got, closed, "q4 x * value * scale")
    dm.close()


@pytest.mark.parametrize("fmt", ["q8", "q4", "f32"])
@pytest.mark.parametrize("cols", [1, 3, 63, 64, 65, 127, 128, 129, 193, 511, 4096])
def test_linear_tails_rows_exact(oracle, srlib, fmt, cols):
    """Exactness across tails and rows (q8_block_test.go:127,
    q4_block_test.go:40): down_proj [64, cols] with quantized random weights,
    subnormal / -0 inputs at fixed strides, every 5th scale 0 and every 11th
    subnormal; rows 1..7 (the 4-row tile and its remainders), 8, 33 and 300
    (the 8-row tiles)."""
    dm = model(hidden=cols, fmt=fmt)
    rng = np.random.default_rng(cols)
    w = (rng.standard_normal((64, cols)) * 0.05).astype(np.float32)
    if fmt == "f32":
        vals, sc = w, None
        dm.load_param(DOWN, w)
    else:
        vals, sc = oracle.quantize(w, Q8 if fmt == "q8" else Q4)
        sc = sc.copy()
        sc[::5] = 0
        sc[::11] = F32_TINY
        dm.load_param(DOWN, vals, sc)
    for rows in (1, 2, 3, 4, 5, 6, 7, 8, 33, 300):
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        flat = x.reshape(-1)
        flat[::13] = F32_TINY
        flat[::17] = np.float32(-0.0)
        flat[5::19] *= np.float32(2.0 ** 60)
        got = dm.linear(DOWN, x)
        f = {"q8": Q8, "q4": Q4, "f32": 0}[fmt]
        want = oracle.linear(x, f, vals, sc if sc is not None else np.zeros(1, np.float32), 64, cols)
        bits_equal(got, want.reshape(got.shape), f"{fmt} cols {cols} rows {rows}")
    dm.close()


def dequant(vals, sc, fmt, rows, cols):
    """Dense fp64 weights from Q8 / Q4 storage (copyRow, M:3900-3921)."""
    g = (cols + 63) // 64
    if fmt == "q8":
        q = vals.view(np.int8).reshape(rows, cols).astype(np.float64)
    else:
        b = vals.view(np.uint8).reshape(rows, (cols + 1) // 2).astype(np.int64)
        nib = np.zeros((rows, 2 * b.shape[1]), dtype=np.int64)
        nib[:, 0::2], nib[:, 1::2] = b & 15, b >> 4
        q = np.where(nib >= 8, nib - 16, nib)[:, :cols].astype(np.float64)
    s = np.repeat(sc.reshape(rows, g).astype(np.float64), 64, axis=1)[:, :cols]
    return q * s


@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("cols", [64, 576, 4096, 14336])
def test_fast_decode_gemv(oracle, srlib, fmt, cols):
    """SR_MODE_FAST projections of 1 and 2 rows run the decode GEMV (128-bit
    code loads, dequantisation in registers): down_proj [64, cols] splits K
    over CTAs (the split-K reduction), gate [cols, 64] and the embedding as a
    head [256, 64] do not.  Each output must be within 1e-5 of sum_j |x_j w_j|
    of the exact-order oracle result (fast mode reorders the fp32 sums)."""
    dm = model(hidden=cols, fmt=fmt)
    rng = np.random.default_rng(cols + (fmt == "q4"))
    for index, (rows_w, cols_w) in ((DOWN, (64, cols)), (7, (cols, 64)), (EMB, (256, 64))):
        w = (rng.standard_normal((rows_w, cols_w)) * 0.05).astype(np.float32)
        vals, sc = oracle.quantize(w, Q8 if fmt == "q8" else Q4)
        dm.load_param(index, vals, sc)
        wd = np.abs(dequant(vals, sc, fmt, rows_w, cols_w))
        for n in (1, 2):
            x = rng.standard_normal((n, cols_w)).astype(np.float32)
            dm.set_mode("exact")
            exact = dm.linear(index, x)
            dm.set_mode("fast")
            got = dm.linear(index, x)
            want = oracle.linear(x, Q8 if fmt == "q8" else Q4, vals, sc, rows_w, cols_w).reshape(got.shape)
            bits_equal(exact, want, f"exact {fmt} param {index} rows {n}")
            bound = np.abs(x).astype(np.float64) @ wd.T
            err = np.abs(got.astype(np.float64) - want) / np.maximum(bound, 1e-30)
            assert err.max() <= 1e-5, (fmt, cols, index, n, float(err.max()))
    dm.close()


@pytest.mark.parametrize("cache", [True, False], ids=["code-cache", "direct-codes"])
@pytest.mark.parametrize("fmt", ["q8", "q4"])
@pytest.mark.parametrize("cols", [64, 576, 4096, 14336])
def test_fast_tensor_core_gemm(oracle, srlib, fmt, cols, cache):
    """SR_MODE_FAST projections of 3 or more rows run the tcgen05 GEMM, with
    the bf16 code cache or (direct) reading the Q8 / Q4 codes as stored and
    widening them to bf16 in shared memory; with the cache, steps of more than
    128 rows run on SM pairs (k_gemm_q2).  down_proj [64, cols]: one
    256-feature tile whose blocks are cut across up to 56 stream-K groups
    (k_sk_reduce adds their partial sums); gate [cols, 64]: many whole tiles,
    the last one partly out of range; the embedding as a head [256, 64].  Row
    counts cover a few rows of one 128-row tile up to four 256-row pair tiles.  Each
    output must be within 3e-5 of sum_j |x_j w_j| of the exact-order oracle
    (bf16 hi + lo activation planes)."""
    dm = model(hidden=cols, fmt=fmt)
    dm.set_mode("fast")
    dm.set_code_cache(cache)
    rng = np.random.default_rng(cols + 7 * (fmt == "q4"))
    for index, (rows_w, cols_w) in ((DOWN, (64, cols)), (7, (cols, 64)), (EMB, (256, 64))):
        w = (rng.standard_normal((rows_w, cols_w)) * 0.05).astype(np.float32)
        vals, sc = oracle.quantize(w, Q8 if fmt == "q8" else Q4)
        dm.load_param(index, vals, sc)
        wd = np.abs(dequant(vals, sc, fmt, rows_w, cols_w))
        for n in (3, 4, 8, 16, 32, 33, 128, 200, 256, 512, 1000):
            x = rng.standard_normal((n, cols_w)).astype(np.float32)
            got = dm.linear(index, x)
            assert dm.code_cache() == cache
            want = oracle.linear(x, Q8 if fmt == "q8" else Q4, vals, sc, rows_w, cols_w, threads=8).reshape(got.shape)
            bound = np.abs(x).astype(np.float64) @ wd.T
            err = np.abs(got.astype(np.float64) - want) / np.maximum(bound, 1e-30)
            assert err.max() <= 3e-5, (fmt, cols, index, n, float(err.max()))
    dm.close()
