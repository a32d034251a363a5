"""Pin the CPU oracle against the reference's Transformers golden fixtures.

Mirrors cmd/monolith/hf_inference_test.go:32-130: for every fixture, prefill
the first 35 ids in chunks of 1/4/16/35 then decode ids 35 and 36, comparing
the returned last-row logits and every layer's K/V with the goldens at abs
tolerance 2e-5; then a ragged two-session prefill + decode batch.
"""

import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, GOLDEN_DIR

# GPT-2 fixtures (hf-gpt2/{legacy-f32,f16,bf16}): the oracle's GPT-2 profile
# (loadGPT2 M:5052-5165, step branches M:6369-6408) against the same goldens.
GPT2 = sorted(glob.glob(os.path.join(GOLDEN_DIR, "gpt2", "*.npz")))

TOL = 2e-5  # hf_inference_test.go: hfNear(..., 2e-5)


def _near(got, want, tol=TOL):
    assert got.shape == want.shape
    assert np.all(np.isfinite(got))
    err = np.abs(got.astype(np.float64) - want.astype(np.float64)).max()
    assert err <= tol, f"max abs error {err:.3g} > {tol}"


@pytest.mark.parametrize("path", GOLDEN + GPT2, ids=lambda p: p.split("/")[-1][:-4])
def test_oracle_matches_transformers(oracle, path):
    m, z, hf = oracle.load_golden(path)
    ids, ref = z["ids"], z["logits"]
    pt = m.cfg.page_tokens
    kd = m.cfg.dim // m.cfg.heads * m.cfg.kv_heads
    pages = 2
    for chunk in (1, 4, 16, 35):
        pool = np.zeros(pages * m.page_elements, dtype=np.float32)
        pos = 0
        for lo in range(0, 35, chunk):
            hi = min(lo + chunk, 35)
            lg = m.step(pool, [pos], [ids[lo:hi]], [list(range(pages))])
            _near(lg[0], ref[hi - 1])
            pos = hi
        for p in (35, 36):
            lg = m.step(pool, [pos], [ids[p:p + 1]], [list(range(pages))])
            _near(lg[0], ref[p])
            pos += 1
        for layer in range(m.cfg.layers):
            for p in range(37):
                base = (p // pt) * m.page_elements + layer * 2 * pt * kd + (p % pt) * kd
                _near(pool[base:base + kd], z["cache_k"][layer, p])
                _near(pool[base + pt * kd:base + pt * kd + kd], z["cache_v"][layer, p])
    # Ragged sessions keep independent positions during shared prefill.
    pool = np.zeros(4 * m.page_elements, dtype=np.float32)
    lg = m.step(pool, [0, 0], [ids[:35], ids[:4]], [[0, 1], [2, 3]])
    _near(lg[0], ref[34])
    _near(lg[1], ref[3])
    lg = m.step(pool, [35, 4], [ids[35:36], ids[4:5]], [[0, 1], [2, 3]])
    _near(lg[0], ref[35])
    _near(lg[1], ref[4])


@pytest.mark.parametrize("page_tokens", [16, 7])
def test_oracle_page_size_invariant(oracle, page_tokens):
    """Logits do not depend on the page size (16-token pages are BASELINE's)."""
    m32, z, hf = oracle.load_golden(GOLDEN[0])
    mp, _, _ = oracle.load_golden(GOLDEN[0], page_tokens=page_tokens)
    ids = z["ids"]
    p32 = np.zeros(2 * m32.page_elements, dtype=np.float32)
    npages = (37 + page_tokens - 1) // page_tokens
    pp = np.zeros(npages * mp.page_elements, dtype=np.float32)
    a = m32.step(p32, [0], [ids[:37]], [[0, 1]])
    b = mp.step(pp, [0], [ids[:37]], [list(range(npages))])
    assert np.array_equal(a, b)


def test_oracle_selected_rows_zeroed(oracle):
    m, z, _ = oracle.load_golden(GOLDEN[0])
    ids = z["ids"]
    pool = np.zeros(4 * m.page_elements, dtype=np.float32)
    lg = m.step(pool, [0, 0], [ids[:5], ids[:3]], [[0], [1]], want_logits=[False, True])
    assert not lg[0].any()
    _near(lg[1], z["logits"][2])


def test_gpt2_fixtures_present():
    assert len(GPT2) == 3


@pytest.mark.parametrize("fmt", ["q8", "q4-mixed"])
def test_oracle_gpt2_quantized_close(oracle, fmt):
    """Quantized GPT-2 storage (the same readParam quantizer on the transposed
    Conv1D matrices, M:5072-5108) stays near the fp32 logits."""
    m32, z, _ = oracle.load_golden(GPT2[0])
    mq, _, _ = oracle.load_golden(GPT2[0], weight_format=fmt)
    ids = z["ids"]
    a = m32.step(np.zeros(2 * m32.page_elements, np.float32), [0], [ids[:37]], [[0, 1]])
    b = mq.step(np.zeros(2 * mq.page_elements, np.float32), [0], [ids[:37]], [[0, 1]])
    err = float(np.abs(a - b).max())
    assert 0 < err < (0.05 if fmt == "q8" else 0.5), err
