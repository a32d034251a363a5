"""Safetensors checkpoint import (sr_go_tranformer_b200.hf) on the CPU.

Checkpoints are rebuilt here from the committed golden fixtures (whose fp32
parameters came from the reference's own testdata safetensors, widened exactly)
and must read back bit for bit in hfProfileSpecs order, single-file and
sharded.  The archive checks of openHFArchiveFormat / readHFConfig
(cmd/monolith/monolith.go:253-385, 644-831) are exercised one mutation at a
time.  When a reference checkout is present, its fixture directories are also
opened directly.
"""

import glob
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN_DIR
from sr_go_tranformer_b200 import hf

DT = {"f32": "F32", "f16": "F16", "bf16": "BF16"}


def _encode(arr, dtype):
    a = np.ascontiguousarray(arr, dtype=np.float32)
    if dtype == "F32":
        return a.astype("<f4").tobytes()
    if dtype == "F16":
        h = a.astype(np.float16)
        assert np.array_equal(h.astype(np.float32), a)
        return h.astype("<f2").tobytes()
    bits = a.view(np.uint32)
    assert np.all(bits & 0xFFFF == 0)
    return (bits >> 16).astype("<u2").tobytes()


def write_safetensors(path, tensors, header_extra=None, order=None, metadata=True, trailing=b""):
    """tensors: {name: (fp32 array, dtype)}; data laid out in `order`."""
    names = order or list(tensors)
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = {"format": "pt"}
    for n in names:
        arr, dt = tensors[n]
        b = _encode(arr, dt)
        header[n] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if header_extra:
        header.update(header_extra)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)
        f.write(trailing)


def fixture_tensors(npz_path):
    z = np.load(npz_path)
    cfg = json.loads(str(z["config"]))
    dt = DT[os.path.basename(npz_path)[:-4].split("-")[-1]]
    h = hf.HFConfig(cfg, 0)
    h.model_type = cfg["model_type"]
    specs = h.specs()
    tensors = {name: (z[f"param_{i}"].reshape(shape), dt) for i, (name, shape) in enumerate(specs)}
    return cfg, tensors, z, specs


def make_checkpoint(d, npz_path, shards=1, seed=0):
    cfg, tensors, z, specs = fixture_tensors(npz_path)
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    names = list(tensors)
    np.random.default_rng(seed).shuffle(names)
    if shards == 1:
        write_safetensors(os.path.join(d, "model.safetensors"), tensors, order=names)
    else:
        parts = np.array_split(np.array(names, dtype=object), shards)
        wm = {}
        for k, part in enumerate(parts):
            fn = f"model-{k + 1:05d}-of-{shards:05d}.safetensors"
            write_safetensors(os.path.join(d, fn), {n: tensors[n] for n in part}, order=list(part))
            wm.update({n: fn for n in part})
        with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": 0}, "weight_map": wm}, f)
    return cfg, tensors, z, specs


FIXTURES = sorted(glob.glob(os.path.join(GOLDEN_DIR, "hf-*.npz")))


@pytest.mark.parametrize("npz", FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
@pytest.mark.parametrize("shards", [1, 3])
def test_archive_reads_fixture_bit_exact(tmp_path, npz, shards):
    _, _, z, specs = make_checkpoint(str(tmp_path), npz, shards)
    a = hf.open_hf_archive(str(tmp_path))
    assert [n for n, _ in a.config.specs()] == [n for n, _ in specs]
    assert len(a.shards) == shards
    for i, (name, _) in enumerate(specs):
        got = a.read_tensor(name)
        want = z[f"param_{i}"]
        assert got.dtype == np.float32
        assert np.array_equal(got.reshape(-1).view(np.uint32), want.reshape(-1).view(np.uint32)), name
    d = a.config.desc("q8", 32)
    cfg = json.loads(str(z["config"]))
    assert (d.vocab, d.dim, d.layers, d.heads, d.kv_heads) == (cfg["vocab_size"], cfg["hidden_size"],
                                                              cfg["num_hidden_layers"], cfg["num_attention_heads"],
                                                              cfg["num_key_value_heads"])
    assert d.context == min(cfg["max_position_embeddings"], 2048)
    assert d.qkv_bias == (cfg["model_type"] == "qwen2")
    assert d.tied == int(cfg.get("tie_word_embeddings", False))


def test_half_float_every_pattern():
    """halfFloat (M:834-847) widens every finite half exactly (IEEE), including
    subnormals and signed zeros; infinities and NaNs keep sign and payload bits."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = hf.half_float(bits).view(np.uint32)
    finite = ((bits >> 10) & 31) != 31
    want = bits.view(np.float16).astype(np.float32).view(np.uint32)
    assert np.array_equal(got[finite], want[finite])
    v = bits[~finite].astype(np.uint32)
    assert np.array_equal(got[~finite], ((v & 0x8000) << 16) | 0x7F800000 | ((v & 1023) << 13))


NPZ = os.path.join(GOLDEN_DIR, "hf-qwen2-untied-bf16.npz")


def _expect_error(tmp_path, mutate, msg, npz=NPZ):
    d = str(tmp_path)
    cfg, tensors, _, specs = make_checkpoint(d, npz)
    mutate(d, cfg, tensors, specs)
    with pytest.raises(hf.HFError, match=msg):
        hf.open_hf_archive(d)


def _rewrite_config(d, cfg):
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)


def _rewrite(d, tensors, **kw):
    write_safetensors(os.path.join(d, "model.safetensors"), tensors, **kw)


def test_rejects_missing_tensor(tmp_path):
    def m(d, cfg, t, specs):
        del t[specs[3][0]]
        _rewrite(d, t)
    _expect_error(tmp_path, m, "missing HF tensor")


def test_rejects_unexpected_tensor(tmp_path):
    def m(d, cfg, t, specs):
        t["model.layers.0.self_attn.rotary_emb.inv_freq"] = (np.ones(4, np.float32), "F32")
        _rewrite(d, t)
    _expect_error(tmp_path, m, "unexpected or duplicate HF tensor")


def test_rejects_shape_mismatch(tmp_path):
    def m(d, cfg, t, specs):
        name = specs[3][0]  # k_proj: [kv_dim, dim], not square
        a, dt = t[name]
        t[name] = (a.T.copy(), dt)
        _rewrite(d, t)
    _expect_error(tmp_path, m, "shape mismatch")


def test_rejects_unsupported_dtype(tmp_path):
    def m(d, cfg, t, specs):
        _rewrite(d, t, header_extra={specs[0][0]: {"dtype": "F64", "shape": list(t[specs[0][0]][0].shape),
                                                     "data_offsets": [0, 8]}})
    _expect_error(tmp_path, m, "dtype/extent")


def test_rejects_trailing_bytes(tmp_path):
    def m(d, cfg, t, specs):
        _rewrite(d, t, trailing=b"\0" * 16)
    _expect_error(tmp_path, m, "trailing/unindexed bytes")


def test_rejects_overlap(tmp_path):
    def m(d, cfg, t, specs):
        names = list(t)
        a0, dt0 = t[names[0]]
        a1, dt1 = t[names[1]]
        n0 = len(_encode(a0, dt0))
        n1 = len(_encode(a1, dt1))
        # second tensor claims bytes that overlap the first one's
        extra = {names[1]: {"dtype": dt1, "shape": list(a1.shape), "data_offsets": [n0 - 2, n0 - 2 + n1]}}
        _rewrite(d, t, header_extra=extra, order=names)
    _expect_error(tmp_path, m, "overlapping|dtype/extent")


def test_rejects_unknown_tensor_field(tmp_path):
    def m(d, cfg, t, specs):
        name = specs[0][0]
        a, dt = t[name]
        n = len(_encode(a, dt))
        _rewrite(d, t, order=list(t), header_extra={
            name: {"dtype": dt, "shape": list(a.shape), "data_offsets": [0, n], "crc": 1}})
    _expect_error(tmp_path, m, "invalid HF tensor header")


def test_rejects_duplicate_json_key(tmp_path):
    def m(d, cfg, t, specs):
        p = os.path.join(d, "config.json")
        txt = open(p).read()
        open(p, "w").write(txt[:-1] + ', "vocab_size": 258}')
    _expect_error(tmp_path, m, "duplicate/invalid JSON key")


def test_rejects_header_not_object(tmp_path):
    def m(d, cfg, t, specs):
        p = os.path.join(d, "model.safetensors")
        raw = bytearray(open(p, "rb").read())
        raw[8] = ord("[")
        open(p, "wb").write(bytes(raw))
    _expect_error(tmp_path, m, "header must start with object")


def test_rejects_non_finite_weight(tmp_path):
    d = str(tmp_path)
    cfg, t, _, specs = make_checkpoint(d, NPZ)
    name = specs[1][0]
    a, dt = t[name]
    a = a.copy()
    a.reshape(-1)[0] = np.inf
    t[name] = (a, dt)
    _rewrite(d, t)
    arc = hf.open_hf_archive(d)  # headers are fine; the value check comes with the read
    with pytest.raises(hf.HFError, match="non-finite HF weight"):
        arc.read_tensor(name)


def test_rejects_bad_shard_index(tmp_path):
    d = str(tmp_path)
    make_checkpoint(d, NPZ, shards=2)
    p = os.path.join(d, "model.safetensors.index.json")
    idx = json.load(open(p))
    k = next(iter(idx["weight_map"]))
    idx["weight_map"][k] = "../" + idx["weight_map"][k]
    json.dump(idx, open(p, "w"))
    with pytest.raises(hf.HFError, match="shard index name/path"):
        hf.open_hf_archive(d)
    del idx["weight_map"][k]
    json.dump(idx, open(p, "w"))
    with pytest.raises(hf.HFError, match="tensor count mismatch"):
        hf.open_hf_archive(d)


def test_rejects_tensor_in_wrong_shard(tmp_path):
    d = str(tmp_path)
    make_checkpoint(d, NPZ, shards=2)
    p = os.path.join(d, "model.safetensors.index.json")
    idx = json.load(open(p))
    files = sorted(set(idx["weight_map"].values()))
    k = next(n for n, f in idx["weight_map"].items() if f == files[0])
    idx["weight_map"][k] = files[1]
    json.dump(idx, open(p, "w"))
    with pytest.raises(hf.HFError, match="unexpected or duplicate HF tensor"):
        hf.open_hf_archive(d)


@pytest.mark.parametrize("edit,msg", [
    (lambda c: c.update(sliding_window=4096), "explicit sliding_window:null"),
    (lambda c: c.pop("sliding_window"), "explicit sliding_window:null"),
    (lambda c: c.update(rope_type="yarn"), "unsupported HF config field"),
    (lambda c: c.update(hidden_act="gelu"), "unsupported HF profile"),
    (lambda c: c.update(architectures=["LlamaForCausalLM"]), "unsupported HF profile"),
    (lambda c: c.update(eos_token_id=None), "scalar BOS/EOS"),
    (lambda c: c.update(bos_token_id=258), "scalar BOS/EOS"),
    (lambda c: c.update(eos_token_id=[2, 3]), "eos_token_id requires"),
    (lambda c: c.update(head_dim=8), "head_dim must equal"),
    (lambda c: c.update(num_attention_heads=5), "divisible"),
    (lambda c: c.update(vocab_size=100), "invalid model dimensions"),
    (lambda c: c.update(rms_norm_eps=0.0), "theta or RMS epsilon"),
    (lambda c: c.update(num_hidden_layers=2.0), "cannot unmarshal"),
])
def test_config_checks_mistral(tmp_path, edit, msg):
    npz = os.path.join(GOLDEN_DIR, "hf-mistral-f16.npz")

    def m(d, cfg, t, specs):
        edit(cfg)
        _rewrite_config(d, cfg)
    _expect_error(tmp_path, m, msg, npz=npz)


def test_config_llama3_rope_and_eos_list(tmp_path):
    npz = os.path.join(GOLDEN_DIR, "hf-llama3-bf16.npz")
    d = str(tmp_path)
    cfg, _, _, _ = make_checkpoint(d, npz)
    cfg["eos_token_id"] = [2, 5, 7]
    _rewrite_config(d, cfg)
    a = hf.open_hf_archive(d)
    assert a.config.eos == 2 and a.config.extra_eos == [5, 7]
    assert a.config.rope == dict(factor=32.0, low=1.0, high=4.0, original=32)
    desc = a.config.desc("f32")
    assert desc.rope_scaling == 1 and desc.rope_factor == 32.0
    for bad in ({"factor": 0.5}, {"rope_type": "linear"}, {"original_max_position_embeddings": 1000},
                {"extra": 1}):
        c2 = json.loads(json.dumps(cfg))
        c2["rope_scaling"].update(bad)
        _rewrite_config(d, c2)
        with pytest.raises(hf.HFError):
            hf.open_hf_archive(d)


def test_context_limit(tmp_path):
    d = str(tmp_path)
    make_checkpoint(d, NPZ)
    assert hf.open_hf_archive(d).config.context == 128
    assert hf.open_hf_archive(d, 64).config.context == 64
    with pytest.raises(hf.HFError, match="context limit"):
        hf.open_hf_archive(d, 129)


# A reference checkout: SR_REFERENCE_ROOT, else a "reference" directory beside this repository.
REF_TESTDATA = os.path.join(os.environ.get("SR_REFERENCE_ROOT") or
                            os.path.join(os.path.dirname(os.path.dirname(GOLDEN_DIR)), "..", "reference"),
                            "testdata")


@pytest.mark.skipif(not os.path.isdir(REF_TESTDATA), reason="no reference checkout")
@pytest.mark.parametrize("npz", FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_reference_fixture_directories(npz):
    """The reference's own fixture directories open and read back as the
    committed fixtures (which tests/golden/make_golden.py made from them)."""
    fam, var = os.path.basename(npz)[:-4].split("-", 2)[1], os.path.basename(npz)[:-4].split("-", 2)[2]
    d = os.path.join(REF_TESTDATA, f"hf-{fam}", var)
    z = np.load(npz)
    a = hf.open_hf_archive(d)
    for i, (name, _) in enumerate(a.config.specs()):
        assert np.array_equal(a.read_tensor(name).reshape(-1).view(np.uint32),
                              z[f"param_{i}"].reshape(-1).view(np.uint32)), name


# ------------------------------------------------------------------ GPT-2 --
GPT2_NPZ = sorted(glob.glob(os.path.join(GOLDEN_DIR, "gpt2", "*.npz")))


def make_gpt2_checkpoint(d, npz_path, prefix=True, masks=False, dtype=None):
    """The inverse of loadGPT2's parameter order: HF Conv1D layout ([in, out]),
    c_attn concatenated, optional "transformer." prefix and legacy masks."""
    z = np.load(npz_path)
    cfg = json.loads(str(z["config"]))
    dt = dtype or DT[os.path.basename(npz_path)[:-4].split("-")[-1]]
    L = cfg["n_layer"]
    P = [z[f"param_{i}"] for i in range(4 + 16 * L)]
    pre = "transformer." if prefix else ""
    t = {pre + "wte.weight": P[0], pre + "wpe.weight": P[1], pre + "ln_f.weight": P[2].reshape(-1),
         pre + "ln_f.bias": P[3].reshape(-1)}
    for i in range(L):
        q = P[4 + 16 * i:4 + 16 * (i + 1)]
        p = f"{pre}h.{i}."
        t[p + "ln_1.weight"], t[p + "ln_1.bias"] = q[0].reshape(-1), q[1].reshape(-1)
        t[p + "attn.c_attn.weight"] = np.concatenate([q[2], q[3], q[4]], 0).T.copy()
        t[p + "attn.c_attn.bias"] = np.concatenate([q[5].reshape(-1), q[6].reshape(-1), q[7].reshape(-1)])
        t[p + "attn.c_proj.weight"], t[p + "attn.c_proj.bias"] = q[8].T.copy(), q[9].reshape(-1)
        t[p + "ln_2.weight"], t[p + "ln_2.bias"] = q[10].reshape(-1), q[11].reshape(-1)
        t[p + "mlp.c_fc.weight"], t[p + "mlp.c_fc.bias"] = q[12].T.copy(), q[13].reshape(-1)
        t[p + "mlp.c_proj.weight"], t[p + "mlp.c_proj.bias"] = q[14].T.copy(), q[15].reshape(-1)
    tensors = {k: (v, dt) for k, v in t.items()}
    if masks:
        n = cfg["n_positions"]
        for i in range(L):
            tensors[f"{pre}h.{i}.attn.bias"] = (np.tril(np.ones((n, n), np.float32)).reshape(1, 1, n, n), "F32")
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    names = list(tensors)
    np.random.default_rng(3).shuffle(names)
    write_safetensors(os.path.join(d, "model.safetensors"), tensors, order=names)
    return cfg, tensors, z


def _params_equal(a, z):
    got = list(a.params())
    assert len(got) == len([k for k in z.files if k.startswith("param_")])
    for i, g in enumerate(got):
        assert np.array_equal(g.reshape(-1).view(np.uint32), z[f"param_{i}"].reshape(-1).view(np.uint32)), i


@pytest.mark.parametrize("npz", GPT2_NPZ, ids=lambda p: os.path.basename(p)[:-4])
@pytest.mark.parametrize("prefix,masks", [(True, False), (False, True)])
def test_gpt2_archive_params_in_loadgpt2_order(tmp_path, npz, prefix, masks):
    _, _, z = make_gpt2_checkpoint(str(tmp_path), npz, prefix, masks)
    a = hf.open_hf_archive(str(tmp_path))
    assert a.config.model_type == "gpt2" and a.config.kv_heads == a.config.heads
    _params_equal(a, z)
    d = a.config.desc("q8", 32)
    cfg = json.loads(str(z["config"]))
    assert (d.arch, d.dim, d.heads, d.kv_heads, d.positions, d.tied) == (1, cfg["n_embd"], cfg["n_head"],
                                                                         cfg["n_head"], cfg["n_positions"], 1)


def test_gpt2_rejects_bad_mask(tmp_path):
    d = str(tmp_path)
    cfg, t, z = make_gpt2_checkpoint(d, GPT2_NPZ[0], prefix=False, masks=True)
    n = cfg["n_positions"]
    t["h.0.attn.bias"] = (np.ones((1, 1, n, n), np.float32), "F32")
    write_safetensors(os.path.join(d, "model.safetensors"), t)
    a = hf.open_hf_archive(d)
    with pytest.raises(hf.HFError, match="legacy causal mask values"):
        list(a.params())
    t["h.0.attn.bias"] = (np.tril(np.ones((n, n), np.float32)).reshape(1, 1, n, n), "F16")
    write_safetensors(os.path.join(d, "model.safetensors"), t)
    with pytest.raises(hf.HFError, match="masks must be F32"):
        hf.open_hf_archive(d)


@pytest.mark.parametrize("edit,msg", [
    (lambda c: c.update(activation_function="gelu"), "unsupported GPT-2 profile"),
    (lambda c: c.update(n_ctx=32), "unsupported GPT-2 profile"),
    (lambda c: c.update(tie_word_embeddings=False), "unsupported GPT-2 profile"),
    (lambda c: c.update(scale_attn_by_inverse_layer_idx=True), "unsupported GPT-2 profile"),
    (lambda c: c.update(rotary_dim=8), "unsupported GPT-2 config field"),
    (lambda c: c.update(n_head=None), "null GPT-2 config field"),
    (lambda c: c.update(eos_token_id=300), "BOS/EOS"),
])
def test_gpt2_config_checks(tmp_path, edit, msg):
    d = str(tmp_path)
    cfg, _, _ = make_gpt2_checkpoint(d, GPT2_NPZ[0])
    edit(cfg)
    _rewrite_config(d, cfg)
    with pytest.raises(hf.HFError, match=msg):
        hf.open_hf_archive(d)


@pytest.mark.skipif(not os.path.isdir(REF_TESTDATA), reason="no reference checkout")
@pytest.mark.parametrize("npz", GPT2_NPZ, ids=lambda p: os.path.basename(p)[:-4])
def test_reference_gpt2_directories(npz):
    var = os.path.basename(npz)[:-4].split("-", 2)[2]
    a = hf.open_hf_archive(os.path.join(REF_TESTDATA, "hf-gpt2", var))
    _params_equal(a, np.load(npz))


@pytest.mark.parametrize("dtype", ["BF16", "F16", "F32"])
def test_threaded_widening_matches_one_thread(tmp_path, dtype):
    """read_tensor widens large tensors in slices on several threads: the
    values equal the one-thread widening bit for bit, and a non-finite value in
    a late slice is still refused."""
    d = str(tmp_path)
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "vocab_size": 70000, "hidden_size": 128,
           "intermediate_size": 64, "num_hidden_layers": 1, "num_attention_heads": 2, "num_key_value_heads": 1,
           "max_position_embeddings": 64, "rope_theta": 1e4, "rms_norm_eps": 1e-5, "hidden_act": "silu",
           "tie_word_embeddings": True, "bos_token_id": 1, "eos_token_id": 2}
    h = hf.HFConfig(cfg, 0)
    h.model_type = "llama"
    rng = np.random.default_rng(5)
    tensors = {}
    for name, shape in h.specs():
        a = (rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * 0.02).reshape(shape)
        if dtype == "BF16":
            a = (a.view(np.uint32) & 0xFFFF0000).view(np.float32)
        elif dtype == "F16":
            a = a.astype(np.float16).astype(np.float32)
        tensors[name] = (a, dtype)
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    write_safetensors(os.path.join(d, "model.safetensors"), tensors)
    a = hf.open_hf_archive(d)
    big = "model.embed_tokens.weight"  # 70000 x 128 = 8.96 M values: three slices
    one = a.read_tensor(big, threads=1)
    many = a.read_tensor(big, threads=4)
    assert np.array_equal(one.view(np.uint32), many.view(np.uint32))
    assert np.array_equal(one, tensors[big][0])
    bad = tensors[big][0].copy()
    bad.reshape(-1)[-5] = np.inf
    tensors[big] = (bad, dtype)
    write_safetensors(os.path.join(d, "model.safetensors"), tensors)
    with pytest.raises(hf.HFError, match="non-finite"):
        hf.open_hf_archive(d).read_tensor(big, threads=4)


@pytest.mark.parametrize("npz", [FIXTURES[0], GPT2_NPZ[1]], ids=["llama", "gpt2"])
def test_load_into_uploads_every_parameter_in_order(tmp_path, npz):
    """load_into (reading ahead on a host thread) hands sr_model_load_param_f32
    every parameter exactly once, in parameter order, with the right values."""
    class Recorder:
        def __init__(self):
            self.calls = []

        def load_param_f32(self, i, values):
            self.calls.append((i, np.array(values, copy=True)))

    if "gpt2" in npz:
        _, _, z = make_gpt2_checkpoint(str(tmp_path), npz)
    else:
        _, _, z, _ = make_checkpoint(str(tmp_path), npz, shards=2)
    rec = Recorder()
    hf.open_hf_archive(str(tmp_path)).load_into(rec)
    n = len([k for k in z.files if k.startswith("param_")])
    assert [i for i, _ in rec.calls] == list(range(n))
    for i, v in rec.calls:
        assert np.array_equal(v.reshape(-1).view(np.uint32), z[f"param_{i}"].reshape(-1).view(np.uint32)), i
