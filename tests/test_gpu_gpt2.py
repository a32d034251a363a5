"""GPU parity of the GPT-2 profile (exact mode) against the oracle and the
reference's three GPT-2 Transformers fixtures.

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


def test_gpt2_refuses_fast_mode_and_synthetic_init(srlib):
    from sr_go_tranformer_b200 import step as S
    import json
    hf = json.loads(str(np.load(GPT2[0])["config"]))
    dm = S.Model(S.desc_from_hf(hf, "q8", 32))
    with pytest.raises(Exception):
        dm.set_mode("fast")
    with pytest.raises(Exception):
        dm.init_synthetic(1)
