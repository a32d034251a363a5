"""Tensor-parallel step on 2 (and 4) GPUs against the single-GPU step.

Each rank holds its shard of the same synthetic model (the counter-based init
generates every rank's part of one full model) and the step all-reduces the
o_proj / down_proj partial sums, over NCCL or over the library's NVLink
peer-memory kernels.  The summation order of those two projections changes, so
logits are compared within the fast-path tolerance; the ranks' logits must be
identical.
"""

import os
import time

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


def exchange_handles(m, rank, size, folder):
    """Every rank's sr_tp_peer_handle through files in `folder` (bounded wait)."""
    tmp = os.path.join(folder, f"h{rank}.tmp")
    with open(tmp, "wb") as f:
        f.write(m.tp_peer_handle())
    os.replace(tmp, os.path.join(folder, f"h{rank}.bin"))
    paths = [os.path.join(folder, f"h{r}.bin") for r in range(size)]
    t0 = time.time()
    while not all(os.path.exists(p) for p in paths):
        assert time.time() - t0 < 120, "peer handles did not arrive"
        time.sleep(0.05)
    return [open(p, "rb").read() for p in paths]


# Uneven head ownership: every KV head replicated on a pair of ranks that
# split its query heads (2/1 at 2 and 4 ranks, 4/3 at 8 ranks: the Qwen2.5-7B
# shape with its real layer dimensions, 2 layers), q/k/v biases, q4-mixed.
UNEVEN = {
    2: dict(vocab=2048, dim=384, hidden=1024, layers=2, heads=3, kv_heads=1, context=1024, rope_theta=1e6,
            tied=False, qkv_bias=True, weight_format="q4-mixed", page_tokens=16),
    4: dict(vocab=2048, dim=768, hidden=2048, layers=2, heads=6, kv_heads=2, context=1024, rope_theta=1e6,
            tied=False, qkv_bias=True, weight_format="q4-mixed", page_tokens=16),
    8: dict(vocab=152064, dim=3584, hidden=18944, layers=2, heads=28, kv_heads=4, context=1024, rope_theta=1e6,
            tied=False, qkv_bias=True, weight_format="q4-mixed", page_tokens=16),
}


def _run(rank, size, nccl_id, mode, q, allreduce="nccl", folder=None, desc=None):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from sr_go_tranformer_b200 import step as S
    d = S.make_desc(**(desc or DESC))
    m = S.Model(d, device=rank, tp_rank=rank, tp_size=size, nccl_id=nccl_id)
    m.init_synthetic(123)
    m.set_mode(mode)
    if allreduce in ("peer", "peer-ll"):
        m.tp_peer_open(exchange_handles(m, rank, size, folder))
        if allreduce == "peer-ll":
            m.tp_peer_set_protocol("ll")
    pool = S.PagePool(m, 128)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 2048, size=n).tolist() for n in (300, 45, 64, 40)]
    caches = [m.new_cache(pool) for _ in prompts]
    outs = [m.prefill_selected(caches, prompts)]
    for _ in range(2):
        toks = [int(np.argmax(x)) for x in outs[-1]]
        outs.append(m.decode_batch(caches, toks))
    pool.close()
    m.close()  # every rank: the peer all-reduce's last barrier
    q.put((rank, outs))


def _tp_logits(size, mode, allreduce="nccl", folder=None, desc=None):
    import multiprocessing as mp
    from sr_go_tranformer_b200 import step as S
    nccl_id = S.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_run, args=(r, size, nccl_id, mode, q, allreduce, folder, desc))
             for r in range(size)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def _single_logits(mode, desc=None):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_run, args=(0, 1, None, mode, q, "nccl", None, desc))
    p.start()
    r = q.get(timeout=600)
    p.join(timeout=120)
    assert p.exitcode == 0
    return r[1]


@pytest.mark.parametrize("allreduce", ["nccl", "peer"])
@pytest.mark.parametrize("size", [2, 4])
@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_tp_matches_single_gpu(mode, size, allreduce, tmp_path):
    if _gpus() < size:
        pytest.skip(f"needs {size} GPUs")
    tp = _tp_logits(size, mode, allreduce, str(tmp_path))
    single = _single_logits(mode)
    for step in range(len(single)):
        b = single[step]
        for r in range(1, size):
            assert np.array_equal(tp[0][step], tp[r][step]), "ranks disagree"  # replicated head, same residual
        err = float(np.abs(tp[0][step] - b).max())
        assert err <= ATOL, f"{mode} step {step}: TP{size} logits differ from 1 GPU by {err:.3g}"
        assert (np.argmax(tp[0][step], 1) == np.argmax(b, 1)).mean() >= 0.75


@pytest.mark.parametrize("size", [2, 4, 8])
@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_tp_uneven_heads_matches_single_gpu(mode, size, tmp_path):
    """KV heads replicated on pairs of ranks with their query heads split
    unevenly (Qwen2.5-7B's 28/4 heads on 8 ranks: 4 and 3 query heads per
    rank), against the same model on one GPU; NCCL all-reduce, and the peer
    kernels at 2 ranks."""
    if _gpus() < size:
        pytest.skip(f"needs {size} GPUs")
    desc = UNEVEN[size]
    single = _single_logits(mode, desc)
    for allreduce in (["nccl", "peer"] if size == 2 else ["nccl"]):
        folder = tmp_path / allreduce
        folder.mkdir()
        tp = _tp_logits(size, mode, allreduce, str(folder), desc)
        for step in range(len(single)):
            b = single[step]
            for r in range(1, size):
                assert np.array_equal(tp[0][step], tp[r][step]), "ranks disagree"
            err = float(np.abs(tp[0][step] - b).max())
            assert err <= ATOL, f"{mode} {allreduce} step {step}: TP{size} logits differ from 1 GPU by {err:.3g}"
            assert (np.argmax(tp[0][step], 1) == np.argmax(b, 1)).mean() >= 0.75


def _absent_rank(rank, q, folder, done):
    """Rank 1 maps the peers but never joins a step; rank 0's step must end with
    SR_ETIMEOUT from its bounded barrier wait (the flag nothing sets)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from sr_go_tranformer_b200 import step as S
    from sr_go_tranformer_b200 import _abi as A
    d = S.make_desc(**DESC)
    nccl_id = open(os.path.join(folder, "nccl_id"), "rb").read()
    m = S.Model(d, device=rank, tp_rank=rank, tp_size=2, nccl_id=nccl_id)
    m.init_synthetic(123)
    m.set_mode("fast")
    m.tp_peer_open(exchange_handles(m, rank, 2, folder))
    code = None
    if rank == 0:
        pool = S.PagePool(m, 16)
        caches = [m.new_cache(pool)]
        t0 = time.time()
        try:
            m.prefill_selected(caches, [[1, 2, 3]])
        except A.SRError as e:
            code = e.code
        elapsed = time.time() - t0
        pool.close()
        done.set()
        q.put((code, elapsed, caches[0].pos))
    else:
        assert done.wait(120)  # stay mapped until rank 0's step has returned
    m.close()


def test_peer_allreduce_absent_rank_times_out(tmp_path):
    """Failure detection without a GPU fault: a rank that never joins makes the
    other's barrier wait expire after its bound; the step reports SR_ETIMEOUT
    and commits nothing."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    from sr_go_tranformer_b200 import step as S
    from sr_go_tranformer_b200 import _abi as A
    with open(tmp_path / "nccl_id", "wb") as f:
        f.write(S.tp_unique_id())
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_absent_rank, args=(r, q, str(tmp_path), done)) for r in range(2)]
    for p in procs:
        p.start()
    code, elapsed, pos = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert code == A.SR_ETIMEOUT
    assert elapsed < 30
    assert pos == 0


@pytest.mark.parametrize("size", [2, 4])
@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_peer_ll_protocol_equals_barrier_protocol(mode, size, tmp_path):
    """SR_PEER_LL sums each chunk in the same rank order as SR_PEER_BARRIER, so
    the logits of every rank must be bit-identical between the two protocols."""
    if _gpus() < size:
        pytest.skip(f"needs {size} GPUs")
    (tmp_path / "a").mkdir()
    (tmp_path / "b").mkdir()
    ll = _tp_logits(size, mode, "peer-ll", str(tmp_path / "a"))
    barrier = _tp_logits(size, mode, "peer", str(tmp_path / "b"))
    for step in range(len(barrier[0])):
        for r in range(size):
            assert np.array_equal(ll[r][step], barrier[r][step]), (step, r)
