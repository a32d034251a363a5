"""Tensor-parallel sharding on the CPU (no GPU needed).

sr_tp_shard is the host-only function that the tensor-parallel constructor uses
to cut every parameter. These tests check three things:
- the shards partition each tensor exactly once, on 64-column block boundaries;
- unsupported head counts are refused;
- 2- and 4-rank gloo forwards that use these shards reproduce the single-rank
  forward, including KV heads replicated on pairs of ranks that split the
  query heads unevenly.

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


QWEN7B = dict(vocab=152064, dim=3584, hidden=18944, layers=2, heads=28, kv_heads=4, context=4096, rope_theta=1e6,
              tied=False, qkv_bias=True, weight_format="q8", page_tokens=16)


def _full_shapes(m):
    """Full parameter shapes in hfProfileSpecs order for a Llama-family desc."""
    hd = m["dim"] // m["heads"]
    kd, d, h, L = hd * m["kv_heads"], m["dim"], m["hidden"], m["layers"]
    full = [(m["vocab"], d)] + [(1, d), (d, d), (kd, d), (kd, d), (d, d), (1, d), (h, d), (h, d), (d, h)] * L
    full += [(1, d)]
    if m.get("qkv_bias"):
        full += [(1, d), (1, kd), (1, kd)] * L
    if not m.get("tied", True):
        full += [(m["vocab"], d)]
    return full


@pytest.mark.parametrize("shape,size", [("mistral", 1), ("mistral", 2), ("mistral", 4), ("mistral", 8),
                                        ("qwen7b", 2), ("qwen7b", 4), ("qwen7b", 8)])
def test_shards_partition_every_parameter(srlib, shape, size):
    """Every parameter is covered the same number of times by the ranks'
    shards: once when it is sharded, size times when replicated, and
    size / kv_heads times for K/V rows replicated on groups of ranks."""
    from sr_go_tranformer_b200 import step as S
    m = MISTRAL if shape == "mistral" else QWEN7B
    d = _desc(**m)
    full = _full_shapes(m)
    for i, (R, Cc) in enumerate(full):
        cover = np.zeros((R, Cc), dtype=np.int8) if R * Cc <= 1 << 26 else None
        rows_seen, cols_seen = [], []
        for r in range(size):
            r0, nr, c0, nc = S.tp_shard(d, r, size, i)
            assert 0 <= r0 and r0 + nr <= R and 0 <= c0 and c0 + nc <= Cc and nr > 0 and nc > 0
            if nc != Cc and R > 1:
                assert c0 % 64 == 0 and nc % 64 == 0, "column shards hold whole scale blocks"
            rows_seen.append((r0, nr))
            cols_seen.append((c0, nc))
            if cover is not None:
                cover[r0:r0 + nr, c0:c0 + nc] += 1
        if cover is not None:
            replicated = all(x == (0, R) for x in rows_seen) and all(x == (0, Cc) for x in cols_seen)
            k = cover.flat[0]
            assert np.all(cover == k), i
            assert k == size if replicated else k in (1, max(1, size // m["kv_heads"])), (i, k)
    with pytest.raises(Exception):
        S.tp_shard(d, 0, size, len(full))


def test_qwen7b_eight_ranks_split_heads_four_three(srlib):
    """Qwen2.5-7B on 8 ranks: KV head g on ranks 2g and 2g+1, which take query
    heads 7g..7g+3 and 7g+4..7g+6; o_proj shards of 512 / 384 columns; FFN
    shards of 2368 rows; q/k/v biases follow their projections."""
    from sr_go_tranformer_b200 import step as S
    d = _desc(**QWEN7B)
    L = QWEN7B["layers"]
    for r in range(8):
        g, sub = r // 2, r % 2
        q0 = (7 * g + (0 if sub == 0 else 4)) * 128
        nq = (4 if sub == 0 else 3) * 128
        assert S.tp_shard(d, r, 8, 2) == (q0, nq, 0, 3584)          # q_proj rows
        assert S.tp_shard(d, r, 8, 3) == (g * 128, 128, 0, 3584)    # k_proj rows
        assert S.tp_shard(d, r, 8, 4) == (g * 128, 128, 0, 3584)    # v_proj rows
        assert S.tp_shard(d, r, 8, 5) == (0, 3584, q0, nq)          # o_proj columns
        assert S.tp_shard(d, r, 8, 7) == (r * 2368, 2368, 0, 3584)  # gate rows
        assert S.tp_shard(d, r, 8, 9) == (0, 3584, r * 2368, 2368)  # down columns
        nb = 1 + 9 * L + 1  # first bias: layer 0's q bias
        assert S.tp_shard(d, r, 8, nb) == (0, 1, q0, nq)
        assert S.tp_shard(d, r, 8, nb + 1) == (0, 1, g * 128, 128)


def test_unsupported_tensor_parallel_shapes(srlib):
    from sr_go_tranformer_b200 import _abi as A
    from sr_go_tranformer_b200 import step as S
    qwen = _desc(**dict(QWEN7B, weight_format="q4-mixed"))
    assert S.tp_shard(qwen, 1, 4, 2) == (896, 896, 0, 3584)  # rank 1's Q rows: 7 heads x 128
    with pytest.raises(A.SRError) as e:  # 16 ranks: FFN shards of 1184 columns are not whole 64-column blocks
        S.tp_shard(qwen, 0, 16, 1)
    assert e.value.code == A.SR_EUNSUPPORTED
    few = _desc(vocab=512, dim=512, hidden=1024, layers=1, heads=4, kv_heads=4, context=256, weight_format="f32")
    with pytest.raises(A.SRError) as e:  # 8 ranks over 4 KV heads of one query head each: a rank without a head
        S.tp_shard(few, 0, 8, 1)
    assert e.value.code == A.SR_EUNSUPPORTED
    smol = _desc(vocab=49152, dim=576, hidden=1536, layers=2, heads=9, kv_heads=3, context=2048)
    with pytest.raises(A.SRError):  # 3 KV heads over 2 ranks: neither divides the other
        S.tp_shard(smol, 0, 2, 1)
    # head_dim 32, 6 query heads per KV head, 4 ranks: 3 heads (96 columns) per rank
    odd = dict(vocab=512, dim=384, hidden=1024, layers=1, heads=12, kv_heads=2, context=256)
    assert S.tp_shard(_desc(**odd, weight_format="f32"), 3, 4, 5) == (0, 384, 288, 96)  # o_proj columns
    with pytest.raises(A.SRError) as e:  # quantized: 96-column shards are not whole 64-column blocks
        S.tp_shard(_desc(**odd, weight_format="q8"), 0, 4, 1)
    assert e.value.code == A.SR_EUNSUPPORTED


# ----------------------------------------------------------- gloo forward --
def _np_forward(params, hf, ids, cos, sin, shards, reduce_fn, bias=False):
    """fp64 prefill of one sequence; params are this rank's shards (with the
    q/k/v biases after the final norm when `bias`)."""
    d, L = hf["hidden_size"], hf["num_hidden_layers"]
    H = hf["num_attention_heads"]
    hd = d // H
    eps = hf.get("rms_norm_eps", 1e-6)
    Hl = shards[2][1] // hd         # local query heads (Q rows / head_dim)
    Hkvl = shards[3][1] // hd
    group = Hl // Hkvl              # local query heads per local KV head
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
        if bias:
            B = params[2 + 9 * L + 3 * l:5 + 9 * L + 3 * l]
            q, k, v = q + B[0], k + B[1], v + B[2]
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


def _worker(rank, size, port, path, q, bias):
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

    logits = _np_forward(params, hf, z["ids"][:20], cos, sin, shards, allreduce, bias)
    q.put((rank, logits))
    dist.destroy_process_group()


@pytest.mark.parametrize("name,size", [("mistral-f32", 2), ("qwen2-f32", 4)])
def test_gloo_forward_matches_single_rank(srlib, name, size):
    """mistral-f32 (6 query / 2 KV heads) on 2 ranks: one KV head and its 3
    query heads per rank.  qwen2-f32 (the same heads, q/k/v biases) on 4 ranks:
    each KV head replicated on a pair of ranks that split its 3 query heads
    2/1 -- the shape of Qwen2.5-7B on 8 ranks."""
    import multiprocessing as mp
    import socket
    path = [g for g in GOLDEN if os.path.basename(g) == f"hf-{name}.npz"][0]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    import json
    from oracle import oracle as O
    from sr_go_tranformer_b200 import step as S
    z = np.load(path)
    hf = json.loads(str(z["config"]))
    desc = S.desc_from_hf(hf, "f32", 32)
    bias = bool(desc.qkv_bias)
    assert bias == (name == "qwen2-f32")
    if size == 4:
        assert [S.tp_shard(desc, r, size, 2)[1] // (hf["hidden_size"] // hf["num_attention_heads"])
                for r in range(size)] == [2, 1, 2, 1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, size, port, path, q, bias)) for r in range(size)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single-rank reference: same code, no sharding
    full = [z[f"param_{i}"].astype(np.float64) for i in range(len([k for k in z.files if k.startswith("param_")]))]
    om, _, _ = O.load_golden(path)
    cos, sin = om.rope_tables()
    params, shards = _shard_params(full, desc, 0, 1)
    ref = _np_forward(params, hf, z["ids"][:20], cos, sin, shards, lambda a: a, bias)
    for r in range(1, size):
        assert np.allclose(got[0], got[r], rtol=0, atol=1e-12)
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
