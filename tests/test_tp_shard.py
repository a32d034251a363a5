"""Tensor-parallel sharding on the CPU (no GPU needed).

sr_tp_shard is the host-only function that the tensor-parallel constructor uses
to cut every parameter. These tests check three things:
- the shards partition each tensor exactly once, on 64-column block boundaries;
- unsupported head counts are refused;
- a 2-rank gloo forward that uses these shards reproduces the single-rank forward.

The gloo forward runs in float64 numpy: each rank holds its Q/K/V/gate/up rows and its O/down
columns, and the ranks sum the partial O and down outputs with torch.distributed.all_reduce.
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN


def _desc(**kw):
    from sr_go_tranformer_b200 import step as S
    return S.make_desc(**kw)


MISTRAL = dict(vocab=32768, dim=4096, hidden=14336, layers=2, heads=32, kv_heads=8, context=4096,
               rope_theta=1e6, tied=False, weight_format="q8", page_tokens=16)


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_shards_partition_every_parameter(srlib, size):
    from sr_go_tranformer_b200 import step as S
    d = _desc(**MISTRAL)
    # full shapes in hfProfileSpecs order (embedding, 2 layers x 9, final norm, head)
    kd = 4096 // 32 * 8
    full = [(32768, 4096)] + [(1, 4096), (4096, 4096), (kd, 4096), (kd, 4096), (4096, 4096), (1, 4096),
                              (14336, 4096), (14336, 4096), (4096, 14336)] * 2 + [(1, 4096), (32768, 4096)]
    for i, (R, Cc) in enumerate(full):
        cover = np.zeros((R, Cc), dtype=np.int8) if R * Cc <= 1 << 26 else None
        rows_seen, cols_seen = [], []
        for r in range(size):
            r0, nr, c0, nc = S.tp_shard(d, r, size, i)
            assert 0 <= r0 and r0 + nr <= R and 0 <= c0 and c0 + nc <= Cc
            if nc != Cc and R > 1:
                assert c0 % 64 == 0 and nc % 64 == 0, "column shards hold whole scale blocks"
            rows_seen.append((r0, nr))
            cols_seen.append((c0, nc))
            if cover is not None:
                cover[r0:r0 + nr, c0:c0 + nc] += 1
        if cover is not None:
            replicated = all(x == (0, R) for x in rows_seen) and all(x == (0, Cc) for x in cols_seen)
            assert np.all(cover == (size if replicated else 1)), i


def test_unsupported_tensor_parallel_shapes(srlib):
    from sr_go_tranformer_b200 import _abi as A
    from sr_go_tranformer_b200 import step as S
    qwen = _desc(vocab=152064, dim=3584, hidden=18944, layers=2, heads=28, kv_heads=4, context=4096,
                 weight_format="q4-mixed")
    with pytest.raises(A.SRError) as e:
        S.tp_shard(qwen, 0, 8, 1)  # 4 KV heads cannot split 8 ways evenly
    assert e.value.code == A.SR_EUNSUPPORTED
    assert S.tp_shard(qwen, 1, 4, 2) == (896, 896, 0, 3584)  # rank 1's Q rows: 7 heads x 128
    smol = _desc(vocab=49152, dim=576, hidden=1536, layers=2, heads=9, kv_heads=3, context=2048)
    with pytest.raises(A.SRError):
        S.tp_shard(smol, 0, 2, 1)


# ----------------------------------------------------------- gloo forward --
def _np_forward(params, hf, ids, cos, sin, shards, reduce_fn):
    """fp64 prefill of one sequence; params are this rank's shards."""
    d, L = hf["hidden_size"], hf["num_hidden_layers"]
    H, Hkv = hf["num_attention_heads"], hf["num_key_value_heads"]
    hd = d // H
    eps = hf.get("rms_norm_eps", 1e-6)
    Hl = shards[2][1] // hd         # local query heads (Q rows / head_dim)
    Hkvl = shards[3][1] // hd
    group = H // Hkv
    T = len(ids)
    x = params[0][ids].astype(np.float64)

    def rms(v, w):
        return v / np.sqrt((v * v).mean(-1, keepdims=True) + eps) * w

    def rope(v, heads):
        v = v.reshape(T, heads, hd).copy()
        half = hd // 2
        c = cos.reshape(-1, half)[:T][:, None, :]
        s = sin.reshape(-1, half)[:T][:, None, :]
        a, b = v[..., :half].copy(), v[..., half:].copy()
        v[..., :half] = a * c - b * s
        v[..., half:] = a * s + b * c
        return v

    for l in range(L):
        P = params[1 + 9 * l:10 + 9 * l]
        nrm = rms(x, P[0])
        q, k, v = nrm @ P[1].T, nrm @ P[2].T, nrm @ P[3].T
        q, k = rope(q, Hl), rope(k, Hkvl)
        v = v.reshape(T, Hkvl, hd)
        att = np.zeros((T, Hl, hd))
        for h in range(Hl):
            kh = h // group
            sc = q[:, h, :] @ k[:, kh, :].T / np.sqrt(hd)
            sc = sc + np.triu(np.full((T, T), -np.inf), 1)
            p = np.exp(sc - sc.max(-1, keepdims=True))
            att[:, h, :] = (p / p.sum(-1, keepdims=True)) @ v[:, kh, :]
        x = x + reduce_fn(att.reshape(T, -1) @ P[4].T)
        nrm = rms(x, P[5])
        g, u = nrm @ P[6].T, nrm @ P[7].T
        x = x + reduce_fn((g / (1 + np.exp(-g)) * u) @ P[8].T)
    x = rms(x, params[1 + 9 * L])
    head = params[0] if hf.get("tie_word_embeddings", False) else params[-1]
    return x[-1] @ head.T


def _shard_params(full, desc, rank, size):
    from sr_go_tranformer_b200 import step as S
    out, shards = [], []
    for i, p in enumerate(full):
        r0, nr, c0, nc = S.tp_shard(desc, rank, size, i)
        p2 = p.reshape(-1, p.shape[-1]) if p.ndim > 1 else p.reshape(1, -1)
        sl = p2[r0:r0 + nr, c0:c0 + nc]
        out.append(sl if p.ndim > 1 else sl.reshape(-1))
        shards.append((r0, nr, c0, nc))
    return out, shards


def _worker(rank, size, port, path, q):
    import json
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    from oracle import oracle as O
    from sr_go_tranformer_b200 import step as S
    z = np.load(path)
    hf = json.loads(str(z["config"]))
    desc = S.desc_from_hf(hf, "f32", 32)
    full = [z[f"param_{i}"].astype(np.float64) for i in range(len([k for k in z.files if k.startswith("param_")]))]
    om, _, _ = O.load_golden(path)
    cos, sin = om.rope_tables()
    params, shards = _shard_params(full, desc, rank, size)

    def allreduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        dist.all_reduce(t)
        return t.numpy()

    logits = _np_forward(params, hf, z["ids"][:20], cos, sin, shards, allreduce)
    q.put((rank, logits))
    dist.destroy_process_group()


def test_two_rank_gloo_forward_matches_single_rank(srlib):
    import multiprocessing as mp
    import socket
    path = [g for g in GOLDEN if "mistral-f32" in g][0]  # 6 heads / 2 KV heads: 2-way split
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single-rank reference: same code, no sharding
    import json
    from oracle import oracle as O
    from sr_go_tranformer_b200 import step as S
    z = np.load(path)
    hf = json.loads(str(z["config"]))
    desc = S.desc_from_hf(hf, "f32", 32)
    full = [z[f"param_{i}"].astype(np.float64) for i in range(len([k for k in z.files if k.startswith("param_")]))]
    om, _, _ = O.load_golden(path)
    cos, sin = om.rope_tables()
    params, shards = _shard_params(full, desc, 0, 1)
    ref = _np_forward(params, hf, z["ids"][:20], cos, sin, shards, lambda a: a)
    assert np.allclose(got[0], got[1], rtol=0, atol=1e-12)
    assert np.abs(got[0] - ref).max() < 1e-9
    # and against the Transformers golden (fp32 reference) within 2e-5
    assert np.abs(got[0] - z["logits"][19]).max() < 2e-5


def test_gpt2_parameter_table_matches_oracle(oracle):
    """The device's GPT-2 parameter table (loadGPT2 order, M:5052-5165) has the
    oracle's shapes, parameter by parameter."""
    import glob
    import json
    import os
    import numpy as np
    from conftest import GOLDEN_DIR
    from sr_go_tranformer_b200 import step as S
    for path in sorted(glob.glob(os.path.join(GOLDEN_DIR, "gpt2", "*.npz"))):
        hf = json.loads(str(np.load(path)["config"]))
        desc = S.desc_from_hf(hf, "q8", 32)
        om = oracle.Model(oracle.config_from_hf(hf, "q8", 32))
        for i in range(om.nparams):
            info = om.param_info(i)
            row0, rows, col0, cols = S.tp_shard(desc, 0, 1, i)
            assert (row0, col0, rows, cols) == (0, 0, info.rows, info.cols), i
        with pytest.raises(Exception):
            S.tp_shard(desc, 0, 1, om.nparams)
        with pytest.raises(Exception):  # one GPU only
            S.tp_shard(desc, 0, 2, 0)


def test_gpt2_description_checks():
    """validate_desc's GPT-2 rules (readGPT2Config's profile, M:446-513): one
    KV head per query head, a tied head, a position table covering the
    context, one GPU; an unknown architecture is refused."""
    from sr_go_tranformer_b200 import step as S
    hf = dict(model_type="gpt2", vocab_size=258, n_embd=24, n_inner=40, n_layer=2, n_head=6, n_positions=64)
    good = S.desc_from_hf(hf, "q8", 32)
    assert S.tp_shard(good, 0, 1, 1) == (0, 64, 0, 24)  # wpe: n_positions rows
    for field, value in (("kv_heads", 2), ("tied", 0), ("qkv_bias", 1), ("positions", 32), ("arch", 7)):
        d = S.desc_from_hf(hf, "q8", 32)
        setattr(d, field, value)
        with pytest.raises(Exception):
            S.tp_shard(d, 0, 1, 0)
