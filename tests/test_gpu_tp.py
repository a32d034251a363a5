"""Tensor-parallel step on 2 (and 4) GPUs against the single-GPU step.

Each rank holds its shard of the same synthetic model (the counter-based init
generates every rank's part of one full model) and the step all-reduces the
o_proj / down_proj partial sums over NCCL.  The summation order of those two
projections changes, so logits are compared within the fast-path tolerance.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 5e-4


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


DESC = dict(vocab=2048, dim=1024, hidden=2048, layers=2, heads=8, kv_heads=4, context=1024, rope_theta=1e6,
            tied=False, weight_format="q8", page_tokens=16)


def _run(rank, size, nccl_id, mode, q):
    from sr_go_tranformer_b200 import step as S
    d = S.make_desc(**DESC)
    m = S.Model(d, device=rank, tp_rank=rank, tp_size=size, nccl_id=nccl_id)
    m.init_synthetic(123)
    m.set_mode(mode)
    pool = S.PagePool(m, 128)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 2048, size=n).tolist() for n in (300, 45, 64, 40)]
    caches = [m.new_cache(pool) for _ in prompts]
    outs = [m.prefill_selected(caches, prompts)]
    for _ in range(2):
        toks = [int(np.argmax(x)) for x in outs[-1]]
        outs.append(m.decode_batch(caches, toks))
    q.put((rank, outs))


def _tp_logits(size, mode):
    import multiprocessing as mp
    from sr_go_tranformer_b200 import step as S
    nccl_id = S.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_run, args=(r, size, nccl_id, mode, q)) for r in range(size)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def _single_logits(mode):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_run, args=(0, 1, None, mode, q))
    p.start()
    r = q.get(timeout=600)
    p.join(timeout=120)
    assert p.exitcode == 0
    return r[1]


@pytest.mark.parametrize("size", [2, 4])
@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_tp_matches_single_gpu(mode, size):
    if _gpus() < size:
        pytest.skip(f"needs {size} GPUs")
    tp = _tp_logits(size, mode)
    single = _single_logits(mode)
    for step in range(len(single)):
        b = single[step]
        for r in range(1, size):
            assert np.array_equal(tp[0][step], tp[r][step]), "ranks disagree"  # replicated head, same residual
        err = float(np.abs(tp[0][step] - b).max())
        assert err <= ATOL, f"{mode} step {step}: TP{size} logits differ from 1 GPU by {err:.3g}"
        assert (np.argmax(tp[0][step], 1) == np.argmax(b, 1)).mean() >= 0.75
