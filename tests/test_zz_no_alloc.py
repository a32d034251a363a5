"""The allocation-free step, sr_step_noalloc, against sr_step (GPU).

sr_step_noalloc is for callers that cannot allocate device memory while they serve, for example
an engine that has reserved nearly all of HBM for its KV page pool up front. Its only scratch, the
split-K attention partials, lives in a 16 MiB array compiled into the library.

Both entry points run through the C ABI on identical batches: a prefill, then a decode, i.e. two
calls in a row. The logits must agree within the fast-path tolerance, because split-K attention
reorders the softmax sums. The allocation-free step is also compared directly with the CPU oracle
(the reference's arithmetic restated) on weights loaded from the oracle, at the same tolerance, with
the K/V rows it writes checked as well. A batch that needs more than 16 MiB of scratch must be
refused without touching the pool.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 5e-4  # the fast-path tolerance of tests/test_gpu_fast.py


def _batch(A, pos, chunks, tables):
    arrs = {
        "pos": np.asarray(pos, dtype=np.int32),
        "toff": np.concatenate([[0], np.cumsum([len(c) for c in chunks])]).astype(np.int32),
        "tok": np.concatenate([np.asarray(c, dtype=np.int32) for c in chunks]).astype(np.int32),
        "poff": np.concatenate([[0], np.cumsum([len(t) for t in tables])]).astype(np.int32),
        "pid": np.concatenate([np.asarray(t, dtype=np.int32) for t in tables]).astype(np.int32),
    }
    b = A.Batch(len(chunks), arrs["pos"].ctypes.data, arrs["toff"].ctypes.data, arrs["tok"].ctypes.data,
                arrs["poff"].ctypes.data, arrs["pid"].ctypes.data, None)
    return b, arrs


def test_noalloc_step_matches_step(srlib):
    from sr_go_tranformer_b200 import _abi as A
    from sr_go_tranformer_b200 import step as S
    desc = S.make_desc(512, 256, 384, 2, 4, 2, 4096, rope_theta=1e5, tied=True, weight_format="q8", page_tokens=32)
    model = S.Model(desc)
    model.init_synthetic(31)
    model.set_mode("exact")
    pool_a, pool_b = S.PagePool(model, 64), S.PagePool(model, 64)
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 512, size=n).tolist() for n in (300, 40, 7)]
    tables = [list(range(0, 11)), list(range(11, 13)), list(range(13, 14))]
    pos = [0, 0, 0]
    V = desc.vocab
    for call in range(2):  # prefill, then one decode token each
        chunks = prompts if call == 0 else [[int(t)] for t in last]
        b, keep = _batch(A, pos, chunks, tables)
        want = np.zeros((3, V), dtype=np.float32)
        got = np.zeros((3, V), dtype=np.float32)
        A.check(srlib.sr_step(model.h, pool_a.h, C.byref(b), want.ctypes.data, None))
        A.check(srlib.sr_step_noalloc(model.h, pool_b.h, C.byref(b), got.ctypes.data))
        assert np.all(np.isfinite(got))
        err = float(np.abs(got - want).max())
        assert err <= ATOL, f"call {call}: allocation-free logits differ by {err:.3g}"
        last = np.argmax(want, axis=1)
        pos = [p + len(c) for p, c in zip(pos, chunks)]


def test_noalloc_step_matches_oracle(oracle, srlib):
    """Two allocation-free calls in a row (ragged prefill, then decode) against
    the oracle's step on the same weights.  The first layer's K/V rows come
    from exact-order kernels only, so they must equal the oracle's bit for bit;
    later layers follow split-K attention and are held to the tolerance."""
    from sr_go_tranformer_b200 import _abi as A
    from sr_go_tranformer_b200 import step as S
    cfg = oracle.make_config(512, 256, 384, 2, 4, 2, 4096, rope_theta=1e5, tied=False, qkv_bias=True,
                             weight_format="q4-mixed", page_tokens=16)
    om = oracle.Model(cfg)
    om.init_synthetic(33, 0.02)
    model = S.Model(S.make_desc(512, 256, 384, 2, 4, 2, 4096, rope_theta=1e5, tied=False, qkv_bias=True,
                                weight_format="q4-mixed", page_tokens=16))
    for i in range(om.nparams):
        vals, sc = om.get_param_raw(i)
        model.load_param(i, vals, sc)
    pool = S.PagePool(model, 64)
    opool = np.zeros(64 * om.page_elements, dtype=np.float32)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 512, size=n).tolist() for n in (520, 33, 1)]
    tables = [list(range(0, 33)), list(range(33, 36)), list(range(36, 37))]
    pos = [0, 0, 0]
    for call in range(2):
        chunks = prompts if call == 0 else [[int(t)] for t in last]
        b, keep = _batch(A, pos, chunks, tables)
        got = np.zeros((3, 512), dtype=np.float32)
        A.check(srlib.sr_step_noalloc(model.h, pool.h, C.byref(b), got.ctypes.data))
        want = om.step(opool, pos, chunks, tables)
        err = float(np.abs(got - want).max())
        assert err <= ATOL, f"call {call}: allocation-free logits differ from the oracle by {err:.3g}"
        assert (np.argmax(got, axis=1) == np.argmax(want, axis=1)).all()
        last = np.argmax(want, axis=1)
        pos = [p + len(c) for p, c in zip(pos, chunks)]
    kd, pt = cfg.dim // cfg.heads * cfg.kv_heads, 16
    for i, t in enumerate(tables):
        for p in range(pos[i]):
            pg, slot = t[p // pt], p % pt
            for layer in range(cfg.layers):
                k, v = pool.read_row(pg, layer, slot)
                base = pg * om.page_elements + layer * 2 * pt * kd + slot * kd
                ok, ov = opool[base:base + kd], opool[base + pt * kd:base + pt * kd + kd]
                if layer == 0:
                    assert np.array_equal(k, ok) and np.array_equal(v, ov), (i, p)
                else:
                    assert max(np.abs(k - ok).max(), np.abs(v - ov).max()) <= ATOL, (i, p, layer)


def test_noalloc_step_rejects_oversized_scratch(srlib):
    from sr_go_tranformer_b200 import _abi as A
    from sr_go_tranformer_b200 import step as S
    desc = S.make_desc(512, 512, 384, 2, 8, 4, 8192, rope_theta=1e5, tied=True, weight_format="q8", page_tokens=32)
    model = S.Model(desc)
    model.init_synthetic(32)
    pool = S.PagePool(model, 256)
    # 1024 rows at positions 7168..8191 cover 15,872 (row, 512-position split) items;
    # x 4 KV heads x 2 query heads x 66 floats = 33.5 MB > 16 MiB
    k0, v0 = pool.read_row(0, 0, 0)
    b, keep = _batch(A, [7168], [[i % 512 for i in range(1024)]], [list(range(256))])
    rc = srlib.sr_step_noalloc(model.h, pool.h, C.byref(b), None)
    assert rc == A.SR_EINVAL
    assert b"16 MiB" in srlib.sr_last_error()
    k1, v1 = pool.read_row(0, 0, 0)
    assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
