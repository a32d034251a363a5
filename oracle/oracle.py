"""ctypes binding for the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: the oracle restates the reference's Go arithmetic
(cmd/monolith/monolith.go) in C so that tests, smoke() and bench.py's CPU
baseline can check or time it.  The product package never imports this file.
"""

import ctypes as C
import json
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

F32, Q8, Q4 = 0, 1, 2
MODEL_F32, MODEL_Q8, MODEL_Q4, MODEL_Q4_MIXED = 0, 1, 2, 3
FORMATS = {"f32": MODEL_F32, "q8": MODEL_Q8, "q4": MODEL_Q4, "q4-mixed": MODEL_Q4_MIXED}


class Config(C.Structure):
    _fields_ = [("vocab", C.c_int32), ("dim", C.c_int32), ("hidden", C.c_int32), ("layers", C.c_int32),
                ("heads", C.c_int32), ("kv_heads", C.c_int32), ("context", C.c_int32),
                ("rope_theta", C.c_double), ("norm_eps", C.c_double), ("tied", C.c_int32),
                ("qkv_bias", C.c_int32), ("weight_format", C.c_int32), ("page_tokens", C.c_int32),
                ("rope_scaling", C.c_int32), ("rope_factor", C.c_double), ("rope_low", C.c_double),
                ("rope_high", C.c_double), ("rope_original", C.c_int32), ("gpt2", C.c_int32),
                ("positions", C.c_int32)]


class ParamInfo(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("format", C.c_int32),
                ("value_bytes", C.c_int64), ("scale_count", C.c_int64)]


class Sampling(C.Structure):
    _fields_ = [("max_tokens", C.c_int32), ("temperature", C.c_double), ("top_k", C.c_int32),
                ("top_p", C.c_double), ("repeat_penalty", C.c_double), ("seed", C.c_uint64)]


def build():
    """Compile liboracle.so with the committed Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        L.or_rng_uint64.restype = C.c_uint64
        L.or_rng_uint64.argtypes = [C.POINTER(C.c_uint64)]
        L.or_rng_float64.restype = C.c_double
        L.or_rng_float64.argtypes = [C.POINTER(C.c_uint64)]
        L.or_rng_intn.restype = C.c_int64
        L.or_rng_intn.argtypes = [C.POINTER(C.c_uint64), C.c_int64]
        L.or_rng_normal.restype = C.c_double
        L.or_rng_normal.argtypes = [C.POINTER(C.c_uint64)]
        L.or_fill_normal.argtypes = [C.POINTER(C.c_uint64), P, C.c_int64, C.c_double]
        L.or_low_bit_scale.restype = C.c_float
        L.or_low_bit_scale.argtypes = [C.c_float, C.c_double]
        L.or_q8_value.restype = C.c_int8
        L.or_q8_value.argtypes = [C.c_float, C.c_float]
        L.or_quantize.argtypes = [P, C.c_int64, C.c_int64, C.c_int, P, P]
        L.or_copy_row.argtypes = [P, P, C.c_int, C.c_int64, C.c_int64, P]
        L.or_linear.argtypes = [P, P, C.c_int64, C.c_int, P, P, C.c_int64, C.c_int64, C.c_int]
        L.or_rmsnorm.argtypes = [P, P, P, C.c_int64, C.c_int64, C.c_double]
        L.or_model_new.restype = P
        L.or_model_new.argtypes = [C.POINTER(Config)]
        L.or_model_free.argtypes = [P]
        L.or_model_param_count.restype = C.c_int32
        L.or_model_param_count.argtypes = [P]
        L.or_model_param_info.argtypes = [P, C.c_int32, C.POINTER(ParamInfo)]
        L.or_model_set_param.argtypes = [P, C.c_int32, P, P]
        L.or_model_get_param.argtypes = [P, C.c_int32, P, P]
        L.or_model_init_synthetic.argtypes = [P, C.c_uint64, C.c_double]
        L.or_model_init_synthetic_mt.argtypes = [P, C.c_uint64, C.c_double, C.c_int]
        L.or_model_rope_cos.restype = P
        L.or_model_rope_cos.argtypes = [P]
        L.or_model_rope_sin.restype = P
        L.or_model_rope_sin.argtypes = [P]
        L.or_page_elements.restype = C.c_int64
        L.or_page_elements.argtypes = [P]
        L.or_step.argtypes = [P, P, C.c_int64, C.c_int32, P, P, P, P, P, P, P, C.c_int]
        L.or_sample.argtypes = [P, C.c_int32, P, C.c_int32, C.POINTER(Sampling), C.POINTER(C.c_uint64),
                                C.c_int32, C.POINTER(C.c_int32)]
        L.or_schedule_tokens.restype = C.c_int32
        L.or_schedule_tokens.argtypes = [C.c_int32, P, P, C.c_int32, C.c_int32, C.c_int32, C.c_int32]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def config_from_hf(hf, weight_format="f32", page_tokens=32, context=None):
    """Translate an HF config.json dict the way readHFConfig does (M:253-385),
    or readGPT2Config (M:446-513) for model_type gpt2."""
    c = Config()
    if hf.get("model_type") == "gpt2":
        c.vocab, c.dim, c.layers = hf["vocab_size"], hf["n_embd"], hf["n_layer"]
        c.hidden = hf.get("n_inner") or 4 * c.dim
        c.heads = c.kv_heads = hf["n_head"]
        c.positions = hf["n_positions"]
        c.context = context or min(c.positions, 2048)
        c.rope_theta, c.norm_eps = 10000.0, float(hf.get("layer_norm_epsilon", 1e-5))
        c.tied, c.qkv_bias, c.gpt2 = 1, 0, 1
        c.weight_format, c.page_tokens = FORMATS[weight_format], page_tokens
        return c
    c.vocab = hf["vocab_size"]
    c.dim = hf["hidden_size"]
    c.hidden = hf["intermediate_size"]
    c.layers = hf["num_hidden_layers"]
    c.heads = hf["num_attention_heads"]
    c.kv_heads = hf.get("num_key_value_heads", c.heads)
    c.context = context or hf.get("max_position_embeddings", 128)
    c.rope_theta = float(hf.get("rope_theta", 10000.0))
    c.norm_eps = float(hf.get("rms_norm_eps", 1e-6))
    c.tied = 1 if hf.get("tie_word_embeddings", False) else 0
    c.qkv_bias = 1 if hf.get("model_type") == "qwen2" else 0
    c.weight_format = FORMATS[weight_format]
    c.page_tokens = page_tokens
    rs = hf.get("rope_scaling")
    if rs:
        c.rope_scaling = 1
        c.rope_factor = float(rs["factor"])
        c.rope_low = float(rs["low_freq_factor"])
        c.rope_high = float(rs["high_freq_factor"])
        c.rope_original = int(rs["original_max_position_embeddings"])
    return c


def make_config(vocab, dim, hidden, layers, heads, kv_heads, context, rope_theta=1e4, norm_eps=1e-5, tied=True,
                qkv_bias=False, weight_format="f32", page_tokens=32):
    c = Config()
    c.vocab, c.dim, c.hidden, c.layers, c.heads, c.kv_heads, c.context = vocab, dim, hidden, layers, heads, kv_heads, context
    c.rope_theta, c.norm_eps = rope_theta, norm_eps
    c.tied, c.qkv_bias = int(tied), int(qkv_bias)
    c.weight_format, c.page_tokens = FORMATS[weight_format], page_tokens
    return c


def quantize(w, fmt):
    """readParam quantizer (M:857-880) -> (values, scales)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    groups = (cols + 63) // 64
    scales = np.zeros(rows * groups, dtype=np.float32)
    if fmt == Q8:
        vals = np.zeros(rows * cols, dtype=np.int8)
    else:
        vals = np.zeros(rows * ((cols + 1) // 2), dtype=np.uint8)
    lib().or_quantize(_p(w), rows, cols, fmt, _p(vals), _p(scales))
    return vals, scales


def linear(x, fmt, values, scales, out, inp, threads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[0]
    y = np.zeros((n, out), dtype=np.float32)
    lib().or_linear(_p(y), _p(x), n, fmt, _p(values), _p(scales), out, inp, threads)
    return y


class Model:
    """Owns an oracle model (weights + RoPE tables) for one config."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.h = lib().or_model_new(C.byref(cfg))
        if not self.h:
            raise ValueError("invalid oracle config")
        self.nparams = lib().or_model_param_count(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_model_free(self.h)
            self.h = None

    def param_info(self, i):
        info = ParamInfo()
        lib().or_model_param_info(self.h, i, C.byref(info))
        return info

    def set_param_f32(self, i, w):
        """Load an fp32 tensor; quantize it first when the param is Q8/Q4."""
        info = self.param_info(i)
        w = np.ascontiguousarray(w, dtype=np.float32).reshape(info.rows, info.cols)
        if info.format == F32:
            lib().or_model_set_param(self.h, i, _p(w), None)
        else:
            vals, scales = quantize(w, info.format)
            lib().or_model_set_param(self.h, i, _p(vals), _p(scales))

    def set_param_raw(self, i, values, scales):
        lib().or_model_set_param(self.h, i, _p(np.ascontiguousarray(values)),
                                 None if scales is None else _p(np.ascontiguousarray(scales)))

    def get_param_raw(self, i):
        info = self.param_info(i)
        if info.format == F32:
            vals = np.zeros(info.rows * info.cols, dtype=np.float32)
            lib().or_model_get_param(self.h, i, _p(vals), None)
            return vals, None
        dt = np.int8 if info.format == Q8 else np.uint8
        vals = np.zeros(info.value_bytes, dtype=dt)
        scales = np.zeros(info.scale_count, dtype=np.float32)
        lib().or_model_get_param(self.h, i, _p(vals), _p(scales))
        return vals, scales

    def init_synthetic(self, seed, scale=0.02, threads=0):
        if threads:
            lib().or_model_init_synthetic_mt(self.h, seed, scale, threads)
        else:
            lib().or_model_init_synthetic(self.h, seed, scale)

    def rope_tables(self):
        hd = self.cfg.dim // self.cfg.heads
        count = self.cfg.context * (hd // 2)
        cos = np.ctypeslib.as_array(C.cast(lib().or_model_rope_cos(self.h), C.POINTER(C.c_float)), (count,)).copy()
        sin = np.ctypeslib.as_array(C.cast(lib().or_model_rope_sin(self.h), C.POINTER(C.c_float)), (count,)).copy()
        return cos, sin

    @property
    def page_elements(self):
        return lib().or_page_elements(self.h)

    def step(self, pool, pos, chunks, page_tables, want_logits=None, threads=1):
        """One prefillSelected call over sessions; returns logits [B, vocab]."""
        B = len(chunks)
        pos = np.asarray(pos, dtype=np.int32)
        toff = np.zeros(B + 1, dtype=np.int32)
        toff[1:] = np.cumsum([len(c) for c in chunks])
        tokens = np.concatenate([np.asarray(c, dtype=np.int32) for c in chunks]).astype(np.int32)
        poff = np.zeros(B + 1, dtype=np.int32)
        poff[1:] = np.cumsum([len(p) for p in page_tables])
        pids = np.concatenate([np.asarray(p, dtype=np.int32) for p in page_tables]).astype(np.int32)
        want = None if want_logits is None else np.asarray(want_logits, dtype=np.uint8)
        logits = np.zeros((B, self.cfg.vocab), dtype=np.float32)
        num_pages = pool.size // self.page_elements
        rc = lib().or_step(self.h, _p(pool), num_pages, B, _p(pos), _p(toff), _p(tokens), _p(poff), _p(pids),
                           _p(want), _p(logits), threads)
        if rc != 0:
            raise ValueError(f"oracle step rejected the batch ({rc})")
        return logits


def load_golden(path, weight_format="f32", page_tokens=32):
    """Build an oracle Model from a tests/golden/*.npz fixture."""
    z = np.load(path)
    hf = json.loads(str(z["config"]))
    cfg = config_from_hf(hf, weight_format=weight_format, page_tokens=page_tokens)
    m = Model(cfg)
    for i in range(m.nparams):
        m.set_param_f32(i, z[f"param_{i}"])
    return m, z, hf


def sample(logits, history, temperature, top_k, top_p, penalty, rng_state, blocked=-1):
    """sampleWithBlocked; returns (id, new_rng_state) or raises on error."""
    s = Sampling(0, temperature, top_k, top_p, penalty, 0)
    st = C.c_uint64(rng_state)
    out = C.c_int32(-1)
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    hist = np.ascontiguousarray(history, dtype=np.int32) if len(history) else np.zeros(1, dtype=np.int32)
    rc = lib().or_sample(_p(lg), lg.size, _p(hist), len(history), C.byref(s), C.byref(st), blocked, C.byref(out))
    if rc != 0:
        raise ValueError(f"sampling error {rc}")
    return out.value, st.value


def schedule_tokens(remaining, budget, chunk, mixed_chunk, start):
    rem = np.asarray(remaining, dtype=np.int32)
    counts = np.zeros(len(rem), dtype=np.int32)
    total = lib().or_schedule_tokens(len(rem), _p(rem), _p(counts), budget, chunk, mixed_chunk, start)
    return counts.tolist(), total


class RNG:
    def __init__(self, state):
        self.state = C.c_uint64(state)

    def uint64(self):
        return lib().or_rng_uint64(C.byref(self.state))

    def float64(self):
        return lib().or_rng_float64(C.byref(self.state))

    def intn(self, n):
        return lib().or_rng_intn(C.byref(self.state), n)

    def normal(self):
        return lib().or_rng_normal(C.byref(self.state))
