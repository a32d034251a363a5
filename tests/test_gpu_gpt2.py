"""GPU parity of the GPT-2 profile against the oracle and the reference's three
GPT-2 Transformers fixtures: exact mode bit for bit, fast mode within a stated
tolerance.

Mirrors hf_inference_test.go:32-130 for `hf-gpt2/{legacy-f32,f16,bf16}`: prefill
the first 35 ids in chunks of 1/4/16/35, decode ids 35 and 36; logits and every
K/V row bit-exact with the oracle, logits within 2e-5 of Transformers.  Also the
quantized storages against the quantized oracle, and the checkpoint path
through hf.py.
"""

import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN_DIR
from test_gpu_step import assert_same, compare_cache_rows

pytestmark = pytest.mark.gpu

GPT2 = sorted(glob.glob(os.path.join(GOLDEN_DIR, "gpt2", "*.npz")))


def _device(om, hf, fmt):
    from sr_go_tranformer_b200 import step as S
    dm = S.Model(S.desc_from_hf(hf, fmt, om.cfg.page_tokens))
    for i in range(om.nparams):
        vals, sc = om.get_param_raw(i)
        dm.load_param(i, vals, sc)
    return dm


@pytest.mark.parametrize("fmt", ["f32", "q8", "q4-mixed"])
@pytest.mark.parametrize("path", GPT2, ids=lambda p: p.split("/")[-1][:-4])
def test_gpt2_exact_matches_oracle(oracle, srlib, path, fmt):
    from sr_go_tranformer_b200 import step as S
    om, z, hf = oracle.load_golden(path, weight_format=fmt)
    dm = _device(om, hf, fmt)
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
            if fmt == "f32":
                assert np.abs(got[0] - ref[hi - 1]).max() <= 2e-5
        for p in (35, 36):
            got = dm.step(cache, int(ids[p]))
            want = om.step(opool, [p], [ids[p:p + 1]], [cache.pages])
            assert_same(got, want[0], f"decode {p}")
        compare_cache_rows(pool, opool, om, cache)
        cache.close()


def test_gpt2_ragged_batch_and_checkpoint(oracle, srlib, tmp_path):
    """Two ragged sessions in one step, and the same model through a rebuilt
    HF checkpoint (hf.load_hf_model) instead of per-parameter loads."""
    from sr_go_tranformer_b200 import hf, step as S
    from test_hf_archive import make_gpt2_checkpoint
    om, z, _ = oracle.load_golden(GPT2[0])
    make_gpt2_checkpoint(str(tmp_path), GPT2[0], prefix=True, masks=False)
    dm, _ = hf.load_hf_model(str(tmp_path), "f32", page_tokens=32)
    ids = z["ids"]
    pool = S.PagePool(dm, 4)
    ca, cb = dm.new_cache(pool), dm.new_cache(pool)
    got = dm.prefill_selected([ca, cb], [ids[:35], ids[:4]])
    opool = np.zeros(4 * om.page_elements, dtype=np.float32)
    want = om.step(opool, [0, 0], [ids[:35], ids[:4]], [ca.pages, cb.pages])
    assert_same(got, want, "ragged prefill")
    got = dm.decode_batch([ca, cb], [int(ids[35]), int(ids[4])])
    want = om.step(opool, [35, 4], [ids[35:36], ids[4:5]], [ca.pages, cb.pages])
    assert_same(got, want, "ragged decode")
    assert np.abs(got[0] - z["logits"][35]).max() <= 2e-5


def test_gpt2_refuses_synthetic_init(srlib):
    from sr_go_tranformer_b200 import step as S
    import json
    hf = json.loads(str(np.load(GPT2[0])["config"]))
    dm = S.Model(S.desc_from_hf(hf, "q8", 32))
    dm.set_mode("fast")  # accepted: the fast GPT-2 step
    with pytest.raises(Exception):
        dm.init_synthetic(1)


# Fast mode: the fast LayerNorm / GELU kernels, the projections with their biases
# on the tensor cores from 3 rows (the decode GEMV below), split-K attention for
# head_dim 64.  Logits within the fast-mode tolerance of the exact oracle.
FAST_ATOL = 5e-4


def _gpt2_fast_pair(oracle, srlib, om, hf, fmt, prompts, chunk, decode_steps):
    from sr_go_tranformer_b200 import step as S
    dm = _device(om, hf, fmt)
    dm.set_mode("fast")
    pt = om.cfg.page_tokens
    pages = sum((len(p) + decode_steps + pt) // pt + 1 for p in prompts)
    pool = S.PagePool(dm, pages)
    opool = np.zeros(pages * om.page_elements, dtype=np.float32)
    caches = [dm.new_cache(pool) for _ in prompts]
    cursor, last, worst = [0] * len(prompts), [0] * len(prompts), 0.0
    while True:
        chunks = [p[cursor[i]:cursor[i] + chunk] if cursor[i] < len(p) else [last[i]] for i, p in enumerate(prompts)]
        pos = [c.pos for c in caches]
        got = dm.prefill_selected(caches, chunks)
        want = om.step(opool, pos, chunks, [c.pages for c in caches], threads=8)
        err = float(np.abs(got - want).max())
        worst = max(worst, err)
        assert err <= FAST_ATOL, f"{fmt}: fast GPT-2 logits differ by {err:.3g} at positions {pos}"
        last = [int(t) for t in want.argmax(axis=1)]
        for i, p in enumerate(prompts):
            if cursor[i] < len(p):
                cursor[i] += len(chunks[i])
        if all(cursor[i] >= len(p) for i, p in enumerate(prompts)):
            decode_steps -= 1
            if decode_steps < 0:
                break
    pool.close()
    dm.close()
    return worst


@pytest.mark.parametrize("fmt", ["q8", "q4-mixed"])
def test_gpt2_fast_synthetic_matches_oracle(oracle, srlib, fmt):
    """A GPT-2-shaped model (n_embd 256, 4 heads of 64, n_inner 1024, 2 layers,
    vocab 512) with seeded random weights: ragged prefill in chunks of 48 (4 to
    147 rows per step, the tensor cores) and decode steps of 4 rows, then of 2
    and 1 rows (the decode GEMV), against the exact oracle."""
    hf = dict(model_type="gpt2", vocab_size=512, n_embd=256, n_inner=1024, n_layer=2, n_head=4, n_positions=1024,
              layer_norm_epsilon=1e-5)
    om = oracle.Model(oracle.config_from_hf(hf, fmt, 16))
    rng = np.random.default_rng(41)
    for i in range(om.nparams):
        info = om.param_info(i)
        shape = (info.rows, info.cols)
        if info.rows == 1:  # LayerNorm weights near 1, biases and norm shifts small
            w = (0.1 * rng.standard_normal(shape)).astype(np.float32)
            if i in (2,) or (i >= 4 and (i - 4) % 16 in (0, 10)):
                w += 1.0
        else:
            w = (0.02 * rng.standard_normal(shape)).astype(np.float32)
        om.set_param_f32(i, w)
    prompts = [rng.integers(0, 512, size=n).tolist() for n in (130, 47, 20, 3)]
    _gpt2_fast_pair(oracle, srlib, om, hf, fmt, prompts, chunk=48, decode_steps=2)
    _gpt2_fast_pair(oracle, srlib, om, hf, fmt, prompts[:2], chunk=48, decode_steps=1)
    _gpt2_fast_pair(oracle, srlib, om, hf, fmt, prompts[3:], chunk=48, decode_steps=1)


@pytest.mark.parametrize("fmt", ["f32", "q8"])
@pytest.mark.parametrize("path", GPT2, ids=lambda p: p.split("/")[-1][:-4])
def test_gpt2_fast_fixtures_match_oracle(oracle, srlib, path, fmt):
    """The reference's GPT-2 fixtures (head_dim 4: the exact attention; f32
    weights: the exact linears) in fast mode: the fast LayerNorm and GELU."""
    om, z, hf = oracle.load_golden(path, weight_format=fmt)
    ids = [int(t) for t in z["ids"]]
    _gpt2_fast_pair(oracle, srlib, om, hf, fmt, [ids[:35], ids[:9]], chunk=16, decode_steps=2)
