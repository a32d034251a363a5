"""GPU parity of SR_MODE_FAST (split-K attention, FFMA norms, tensor-core
projections) against the CPU oracle within a stated tolerance.

Fast mode reorders fp32 sums (online softmax over split-K attention splits, FMA
contraction, bf16x2-split tensor-core products), so logits are compared with
an absolute tolerance of FAST_ATOL on logits of magnitude ~1 and greedy ids
must agree except on recorded near-ties (margin below FAST_TIE).
"""

import ctypes as C

import numpy as np
import pytest

from test_gpu_step import device_from_oracle

pytestmark = pytest.mark.gpu

FAST_ATOL = 5e-4
FAST_TIE = 2 * FAST_ATOL


def run_pair(oracle, srlib, om, prompts, chunk, decode_steps, threads=8, cache=True):
    from sr_go_tranformer_b200 import step as S
    dm = device_from_oracle(om, srlib, mode="fast")
    dm.set_code_cache(cache)
    pages = sum((len(p) + decode_steps + om.cfg.page_tokens) // om.cfg.page_tokens + 1 for p in prompts)
    pool = S.PagePool(dm, pages)
    opool = np.zeros(pages * om.page_elements, dtype=np.float32)
    caches = [dm.new_cache(pool) for _ in prompts]
    cursor = [0] * len(prompts)
    worst, ties = 0.0, 0
    last = [None] * len(prompts)
    while True:
        chunks, want = [], []
        for i, p in enumerate(prompts):
            if cursor[i] < len(p):
                chunks.append(p[cursor[i]:cursor[i] + chunk])
            else:
                chunks.append([last[i]])
            want.append(cursor[i] + len(chunks[-1]) >= len(p))
        pos = [c.pos for c in caches]
        got = dm.prefill_selected(caches, chunks, want)
        exp = om.step(opool, pos, chunks, [c.pages for c in caches], want, threads=threads)
        err = float(np.abs(got - exp).max())
        worst = max(worst, err)
        assert err <= FAST_ATOL, f"fast logits differ by {err:.3g} at positions {pos}"
        for i in range(len(prompts)):
            if want[i]:
                a, b = int(np.argmax(got[i])), int(np.argmax(exp[i]))
                if a != b:
                    srt = np.sort(exp[i])
                    assert srt[-1] - srt[-2] < FAST_TIE, "greedy id differs without a near-tie"
                    ties += 1
                last[i] = b
            if cursor[i] < len(prompts[i]):
                cursor[i] += len(chunks[i])
        if all(cursor[i] >= len(prompts[i]) for i in range(len(prompts))):
            decode_steps -= 1
            if decode_steps < 0:
                break
    return worst, ties


def test_fast_smollm_shape_long_contexts(oracle, srlib):
    """hd 64, 3 query heads per KV head; contexts up to 700 (3 splits)."""
    cfg = oracle.make_config(4096, 576, 1536, 2, 9, 3, 1024, rope_theta=1e5, tied=True, weight_format="q8",
                             page_tokens=16)
    om = oracle.Model(cfg)
    om.init_synthetic(3, 0.02)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 4096, size=n).tolist() for n in (700, 300, 65, 9)]
    worst, ties = run_pair(oracle, srlib, om, prompts, chunk=256, decode_steps=3)
    assert worst <= FAST_ATOL


@pytest.mark.parametrize("cache", [True, False], ids=["code-cache", "direct-codes"])
def test_fast_mistral_shape_one_layer(oracle, srlib, cache):
    """hd 128, 4 query heads per KV head, Q8; contexts up to 600; with the bf16
    code cache and with the codes read as stored."""
    cfg = oracle.make_config(2048, 4096, 14336, 1, 32, 8, 1024, rope_theta=1e6, tied=False, weight_format="q8",
                             page_tokens=16)
    om = oracle.Model(cfg)
    om.init_synthetic(5, 0.02)
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, 2048, size=n).tolist() for n in (600, 257, 31)]
    worst, ties = run_pair(oracle, srlib, om, prompts, chunk=300, decode_steps=2, cache=cache)
    assert worst <= FAST_ATOL


def test_fast_qwen_shape_bias_q4(oracle, srlib):
    """hd 128, 7 query heads per KV head, QKV bias, q4-mixed."""
    cfg = oracle.make_config(1024, 896, 1024, 1, 7, 1, 1024, rope_theta=1e6, tied=False, qkv_bias=True,
                             weight_format="q4-mixed", page_tokens=32)
    om = oracle.Model(cfg)
    om.init_synthetic(8, 0.02)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, 1024, size=n).tolist() for n in (520, 40)]
    worst, ties = run_pair(oracle, srlib, om, prompts, chunk=200, decode_steps=2)
    assert worst <= FAST_ATOL


def test_fast_qwen_shape_32k_context_decode(oracle, srlib):
    """Config 5's attention shape (hd 128, 7 query heads per KV head, QKV bias,
    q4-mixed) at the full 32,768-token context: one decode step whose rows read
    32,000 / 20,000 / 777 earlier positions (up to 63 attention splits), with
    the same K/V pages on both sides (filled synthetically on the device, read
    back for the oracle: a 32K-token CPU prefill would take minutes)."""
    from sr_go_tranformer_b200 import step as S
    pt = 16
    cfg = oracle.make_config(512, 896, 512, 1, 7, 1, 32768, rope_theta=1e6, tied=False, qkv_bias=True,
                             weight_format="q4-mixed", page_tokens=pt)
    om = oracle.Model(cfg)
    om.init_synthetic(12, 0.02)
    dm = device_from_oracle(om, srlib, mode="fast")
    pos = [32000, 20000, 777]
    npages = sum((p + 1 + pt - 1) // pt for p in pos)
    pool = S.PagePool(dm, npages)
    pool.fill_synthetic(77, 0.5)
    opool = np.zeros(npages * om.page_elements, dtype=np.float32)
    kd = dm.kv_dim
    caches = []
    for p in pos:
        c = dm.new_cache(pool)
        c.ensure_pages(p + 1)
        for q in range(p):  # the oracle sees the same earlier rows
            pg, slot = c.pages[q // pt], q % pt
            k, v = pool.read_row(pg, 0, slot)
            base = pg * om.page_elements + slot * kd
            opool[base:base + kd] = k
            opool[base + pt * kd:base + pt * kd + kd] = v
        c.pos = p
        caches.append(c)
    rng = np.random.default_rng(4)
    chunks = [[int(t)] for t in rng.integers(0, 512, size=len(pos))]
    got = dm.prefill_selected(caches, chunks, [True] * len(pos))
    exp = om.step(opool, pos, chunks, [c.pages for c in caches], [True] * len(pos), threads=8)
    err = float(np.abs(got - exp).max())
    assert err <= FAST_ATOL, f"32K-context decode logits differ by {err:.3g}"


@pytest.mark.parametrize("rows", [1, 2, 4, 16, 31])
def test_fast_decode_rows(oracle, srlib, rows):
    """Fast-mode decode steps of 1, 4, 16 and 31 rows (the decode GEMV at 1
    row, the tensor cores from 3) on the Mistral-7B layer shape, 2 layers, Q8:
    `rows` sessions with short prompts, then 3 decode steps, each against the
    oracle."""
    cfg = oracle.make_config(2048, 4096, 14336, 2, 32, 8, 512, rope_theta=1e6, tied=False, weight_format="q8",
                             page_tokens=16)
    om = oracle.Model(cfg)
    om.init_synthetic(21, 0.02, threads=8)
    rng = np.random.default_rng(22 + rows)
    prompts = [rng.integers(0, 2048, size=int(rng.integers(1, 4))).tolist() for _ in range(rows)]
    worst, ties = run_pair(oracle, srlib, om, prompts, chunk=4, decode_steps=3)
    assert worst <= FAST_ATOL


def _launches(dm):
    from sr_go_tranformer_b200 import _abi as A
    ms = (C.c_double * len(A.PROF_CLASSES))()
    la = (C.c_int64 * len(A.PROF_CLASSES))()
    span, steps, total = C.c_double(), C.c_int64(), C.c_int64()
    A.check(A.lib().sr_profile_read(dm.h, ms, la, C.byref(span), C.byref(steps), C.byref(total), 1))
    return total.value


@pytest.mark.parametrize("shape", ["decode", "ragged"])
def test_split_step_matches_oracle_and_whole_step(oracle, srlib, shape):
    """Split steps: a fast-mode step whose rows can be cut at a session boundary
    into two halves of 64..512 rows runs as two halves on two SM partitions.
    Mistral-7B layer shape, 2 layers, Q8.  "decode": 130 sessions with short
    prompts, then 2 decode steps of 130 rows (halves of 65).  "ragged": prefill
    chunks of 300, 120 and 40 rows beside 140 one-row sessions.  Each step's
    logits are checked against the oracle and against the same model stepping
    whole (split off), and the split model must launch more kernels (each half
    launches its own)."""
    from sr_go_tranformer_b200 import step as S
    cfg = oracle.make_config(2048, 4096, 14336, 2, 32, 8, 1024, rope_theta=1e6, tied=False, weight_format="q8",
                             page_tokens=16)
    om = oracle.Model(cfg)
    om.init_synthetic(31, 0.02, threads=8)
    rng = np.random.default_rng(32 if shape == "decode" else 33)
    if shape == "decode":
        prompts = [rng.integers(0, 2048, size=int(rng.integers(1, 4))).tolist() for _ in range(130)]
    else:
        prompts = [rng.integers(0, 2048, size=n).tolist() for n in (300, 120, 40)] + \
                  [rng.integers(0, 2048, size=1).tolist() for _ in range(140)]
    models = []
    for split in (True, False):
        dm = device_from_oracle(om, srlib, mode="fast")
        dm.set_split(split)
        pages = sum((len(p) + 3 + 16) // 16 + 1 for p in prompts)
        pool = S.PagePool(dm, pages)
        models.append((dm, pool, [dm.new_cache(pool) for _ in prompts]))
    opool = np.zeros(sum((len(p) + 3 + 16) // 16 + 1 for p in prompts) * om.page_elements, dtype=np.float32)
    ocaches = models[1][2]  # page tables match: both pools hand out pages in the same order
    chunks = prompts
    launches = []
    for step in range(3):
        pos = [c.pos for c in ocaches]
        got = [dm.prefill_selected(caches, chunks) for dm, _, caches in models]
        launches.append([_launches(dm) for dm, _, _ in models])
        want = om.step(opool, pos, chunks, [c.pages for c in ocaches], threads=8)
        for g in got:
            err = float(np.abs(g - want).max())
            assert err <= FAST_ATOL, f"step {step}: split-step logits differ from the oracle by {err:.3g}"
        assert float(np.abs(got[0] - got[1]).max()) <= FAST_ATOL
        chunks = [[int(t)] for t in want.argmax(axis=1)]
    assert all(a > b for a, b in launches), launches
    for dm, pool, _ in models:
        pool.close()
        dm.close()
