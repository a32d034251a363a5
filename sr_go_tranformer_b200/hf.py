"""Hugging Face Safetensors checkpoints into a device model.

Restates the reference's HF import (cmd/monolith/monolith.go, "M:line") for the
Llama / Qwen2 / full-attention Mistral profiles the step runs:

* read_hf_config      readHFConfig (M:253-385): bounded, duplicate-free JSON,
                      an allow-list of fields, the profile checks and the
                      context cap (the model maximum, at most 2048 by default);
* open_hf_archive     openHFArchiveFormat (M:644-831): one model.safetensors or
                      a model.safetensors.index.json with shards; every header
                      is checked (names and shapes of hfProfileSpecs M:407-442,
                      dtype widths, extents, no gaps, overlaps or trailing
                      bytes) before any weight is read;
* HFArchive.read_tensor  readTensorValues (M:856-894): F32 / BF16 / F16 widened
                      to fp32 exactly (halfFloat M:834-847), non-finite values
                      rejected; one tensor at a time from a memory map, so the
                      full fp32 model is never held on the host;
* HFArchive.load_into streams the tensors, in parameter order, into
                      sr_model_load_param_f32, which quantizes on the device with
                      the reference's block quantizer (readParam M:857-880); a
                      tensor-parallel rank keeps its shard of each full tensor.

GPT-2 archives (readGPT2Config M:446-513, gpt2Specs M:515-530) open and read
the same way; HFArchive.params() gives their tensors in loadGPT2's parameter
order (M:5052-5165: Conv1D weights transposed to [out, in], c_attn split into
q, k, v), with the legacy causal masks checked.  The device runs GPT-2 in the
exact mode only.

Errors raise HFError with the reference's messages.
"""

import json
import os

import numpy as np

MAX_HF_HEADER = 4 << 20          # maxHFHeader (M:123)
MAX_HF_VOCAB = 262144            # maxHFVocab (M:49)
MAX_HF_PARAMETERS = 8_000_000_000  # maxHFParameters (M:48)
MAX_ACTIVATION_ELEMENTS = 128 * 1024 * 1024  # maxActivationElements (M:50)
BASE_VOCAB = 258                 # baseVocab (M:46)
WIDTH = {"F32": 4, "F16": 2, "BF16": 2}  # hfWidth (M:634-642)

_ALLOWED = ("architectures model_type vocab_size hidden_size intermediate_size num_hidden_layers "
            "num_attention_heads num_key_value_heads max_position_embeddings rope_theta rms_norm_eps hidden_act "
            "tie_word_embeddings attention_bias mlp_bias rope_interleaved attention_dropout pretraining_tp "
            "bos_token_id eos_token_id pad_token_id initializer_range is_llama_config torch_dtype dtype "
            "transformers_version transformers.js_config use_cache _name_or_path _attn_implementation").split()
_ARCH = {"llama": "LlamaForCausalLM", "qwen2": "Qwen2ForCausalLM", "mistral": "MistralForCausalLM"}
_GPT2_ALLOWED = ("architectures model_type vocab_size n_embd n_inner n_layer n_head n_positions n_ctx "
                 "layer_norm_epsilon activation_function scale_attn_weights scale_attn_by_inverse_layer_idx "
                 "reorder_and_upcast_attn add_cross_attention tie_word_embeddings bos_token_id eos_token_id "
                 "pad_token_id attn_pdrop resid_pdrop embd_pdrop initializer_range torch_dtype dtype "
                 "transformers_version use_cache _name_or_path _attn_implementation summary_type summary_use_proj "
                 "summary_activation summary_proj_to_labels summary_first_dropout task_specific_params").split()


class HFError(ValueError):
    pass


# ------------------------------------------------------------------ JSON --
def unique_json(data):
    """uniqueJSON (M:176-228): valid UTF-8, no duplicate keys, depth <= 32,
    at most 2,000,000 nodes, no trailing document."""
    if isinstance(data, (bytes, bytearray)):
        try:
            text = bytes(data).decode("utf-8")
        except UnicodeDecodeError:
            raise HFError("invalid JSON UTF-8")
    else:
        text = data

    def pairs(kv):
        d = {}
        for k, v in kv:
            if k in d:
                raise HFError(f"duplicate/invalid JSON key {k}")
            d[k] = v
        return d

    try:
        value = json.loads(text, object_pairs_hook=pairs, parse_constant=_reject_constant)
    except HFError:
        raise
    except json.JSONDecodeError as e:
        raise HFError("trailing JSON data" if e.msg == "Extra data" else f"invalid JSON: {e.msg}")
    nodes = 0
    stack = [(value, 0)]
    while stack:
        v, depth = stack.pop()
        nodes += 1
        if depth > 32 or nodes > 2_000_000:
            raise HFError("JSON complexity limit")
        if isinstance(v, dict):
            stack.extend((x, depth + 1) for x in v.values())
        elif isinstance(v, list):
            stack.extend((x, depth + 1) for x in v)
    return value


def _reject_constant(name):
    raise HFError(f"invalid JSON: {name}")


def read_bounded_json(path, limit):
    """readBoundedJSON (M:230-250): a regular file of at most `limit` bytes."""
    if not os.path.isfile(path) or os.path.getsize(path) > limit:
        raise HFError(f"{os.path.basename(path)}: metadata size/type limit")
    with open(path, "rb") as f:
        return unique_json(f.read(limit + 1))


# ---------------------------------------------------------------- config --
def _is_int(v):
    return isinstance(v, int) and not isinstance(v, bool)


def _field(raw, key, kind, default):
    """Go's json.Unmarshal into a typed field: absent or null keeps the zero value,
    a value of another JSON type is an error."""
    v = raw.get(key)
    if v is None:
        return default
    ok = {"int": _is_int(v), "float": (_is_int(v) or isinstance(v, float)), "bool": isinstance(v, bool),
          "str": isinstance(v, str), "strs": isinstance(v, list) and all(isinstance(x, str) for x in v)}[kind]
    if not ok:
        raise HFError(f"json: cannot unmarshal {type(v).__name__} into field {key}")
    return float(v) if kind == "float" else v


class HFConfig:
    """The checked HF config (hfConfig, M:134-160) and the step Config (M:56-66)."""

    def __init__(self, raw, context):
        f = lambda k, kind, d: _field(raw, k, kind, d)  # noqa: E731
        self.raw = raw
        self.model_type = f("model_type", "str", "")
        self.architectures = f("architectures", "strs", [])
        self.vocab = f("vocab_size", "int", 0)
        self.dim = f("hidden_size", "int", 0)
        self.hidden = f("intermediate_size", "int", 0)
        self.layers = f("num_hidden_layers", "int", 0)
        self.heads = f("num_attention_heads", "int", 0)
        self.kv_heads = f("num_key_value_heads", "int", 0)
        self.max_positions = f("max_position_embeddings", "int", 0)
        self.theta = f("rope_theta", "float", 0.0)
        self.eps = f("rms_norm_eps", "float", 0.0)
        self.tied = f("tie_word_embeddings", "bool", False)
        self.bos = f("bos_token_id", "int", 0)
        self.eos = 0
        self.extra_eos = []
        self.rope = None
        self.context = context
        self.positions = self.max_positions  # wpe rows (GPT-2)

    @property
    def kv_dim(self):
        return self.dim // self.heads * self.kv_heads

    def parameter_count(self):
        """hfParameterCount (M:387-398)."""
        d, h, k, l = self.dim, self.hidden, self.kv_dim, self.layers
        if self.model_type == "gpt2":
            return (self.vocab + self.positions) * d + l * (4 * d * d + 2 * d * h + 9 * d + h) + 2 * d
        n = self.vocab * d + l * (2 * d + 2 * d * d + 2 * d * k + 3 * d * h) + d
        if self.model_type == "qwen2":
            n += l * (d + 2 * k)
        if not self.tied:
            n += self.vocab * d
        return n

    def specs(self):
        """hfProfileSpecs (M:407-442): (name, shape) in parameter order; for
        GPT-2 the archive's tensors (gpt2Specs, M:515-530)."""
        d, k, h, L = self.dim, self.kv_dim, self.hidden, self.layers
        if self.model_type == "gpt2":
            out = [("wte.weight", (self.vocab, d)), ("wpe.weight", (self.positions, d)), ("ln_f.weight", (d,)),
                   ("ln_f.bias", (d,))]
            for i in range(L):
                p = f"h.{i}."
                out += [(p + "ln_1.weight", (d,)), (p + "ln_1.bias", (d,)), (p + "attn.c_attn.weight", (d, 3 * d)),
                        (p + "attn.c_attn.bias", (3 * d,)), (p + "attn.c_proj.weight", (d, d)),
                        (p + "attn.c_proj.bias", (d,)), (p + "ln_2.weight", (d,)), (p + "ln_2.bias", (d,)),
                        (p + "mlp.c_fc.weight", (d, h)), (p + "mlp.c_fc.bias", (h,)),
                        (p + "mlp.c_proj.weight", (h, d)), (p + "mlp.c_proj.bias", (d,))]
            return out
        out = [("model.embed_tokens.weight", (self.vocab, d))]
        for i in range(L):
            p = f"model.layers.{i}."
            out += [(p + "input_layernorm.weight", (d,)), (p + "self_attn.q_proj.weight", (d, d)),
                    (p + "self_attn.k_proj.weight", (k, d)), (p + "self_attn.v_proj.weight", (k, d)),
                    (p + "self_attn.o_proj.weight", (d, d)), (p + "post_attention_layernorm.weight", (d,)),
                    (p + "mlp.gate_proj.weight", (h, d)), (p + "mlp.up_proj.weight", (h, d)),
                    (p + "mlp.down_proj.weight", (d, h))]
        out.append(("model.norm.weight", (d,)))
        if self.model_type == "qwen2":
            for i in range(L):
                p = f"model.layers.{i}.self_attn."
                out += [(p + "q_proj.bias", (d,)), (p + "k_proj.bias", (k,)), (p + "v_proj.bias", (k,))]
        if not self.tied:
            out.append(("lm_head.weight", (self.vocab, d)))
        return out

    def optional(self):
        """Legacy GPT-2 causal masks (M:693-701): accepted, F32 only, when small."""
        if self.model_type != "gpt2" or self.positions * self.positions * self.layers > MAX_ACTIVATION_ELEMENTS:
            return {}
        return {f"h.{i}.attn.bias": (1, 1, self.positions, self.positions) for i in range(self.layers)}

    def canonical(self, name):
        """GPT-2 archives may prefix every tensor with "transformer." (M:687-692)."""
        return name[len("transformer."):] if self.model_type == "gpt2" and name.startswith("transformer.") else name

    def desc(self, weight_format="f32", page_tokens=32):
        """sr_model_desc of this profile (readHFConfig's Config plus the RoPE scaling;
        for GPT-2 the position table, exact mode only on the device)."""
        from .step import desc_from_hf
        if self.model_type == "gpt2":
            return desc_from_hf(self.raw, weight_format, page_tokens, context=self.context)
        hf = dict(self.raw)
        hf["num_key_value_heads"] = self.kv_heads
        return desc_from_hf(hf, weight_format, page_tokens, context=self.context)


def read_hf_config(path, context_limit=0):
    """readHFConfig (M:253-385) for config.json in directory `path`."""
    raw = read_bounded_json(os.path.join(path, "config.json"), 1 << 20)
    if not isinstance(raw, dict):
        raise HFError("invalid HF config")
    mt = raw.get("model_type")
    if not isinstance(mt, str):
        raise HFError("invalid HF model_type")
    if mt == "gpt2":
        return read_gpt2_config(raw, context_limit)
    keys = set(_ALLOWED)
    if mt == "qwen2":
        keys |= {"use_sliding_window", "sliding_window", "max_window_layers", "layer_types"}
    if mt == "llama":
        keys |= {"head_dim", "rope_scaling"}
    if mt == "mistral":
        keys |= {"head_dim", "sliding_window"}
        if "sliding_window" not in raw or raw["sliding_window"] is not None:
            raise HFError("Mistral requires explicit sliding_window:null; sliding attention is not supported")
    for k, v in raw.items():
        if k == "rope_scaling" and v is None:
            continue
        if k not in keys:
            raise HFError(f'unsupported HF config field "{k}"')
    extra = []
    eos = raw.get("eos_token_id")
    if isinstance(eos, list):
        if mt != "llama" or not 1 <= len(eos) <= 8:
            raise HFError("Llama eos_token_id requires 1..8 integer IDs")
        seen = set()
        for i, v in enumerate(eos):
            if not _is_int(v) or v < 0 or v in seen:
                raise HFError("Llama eos_token_id contains an invalid or duplicate ID")
            seen.add(v)
            if i > 0:
                extra.append(v)
        eos = eos[0]
    h = HFConfig(raw, 0)
    h.eos = _field({"e": eos}, "e", "int", 0)
    h.extra_eos = extra
    for k, kind in (("hidden_act", "str"), ("attention_bias", "bool"), ("mlp_bias", "bool"),
                    ("rope_interleaved", "bool"), ("attention_dropout", "float"), ("pretraining_tp", "int"),
                    ("use_sliding_window", "bool"), ("layer_types", "strs"), ("head_dim", "int")):
        _field(raw, k, kind, None)
    for e in extra:
        if e >= h.vocab:
            raise HFError("Llama EOS ID outside vocabulary")
    if "head_dim" in raw and (raw["head_dim"] is None or h.heads < 1 or h.dim % h.heads != 0 or
                              raw["head_dim"] != h.dim // h.heads):
        raise HFError("HF head_dim must equal hidden_size / num_attention_heads")
    rs = raw.get("rope_scaling")
    if rs is not None:
        if not isinstance(rs, dict):
            raise HFError("invalid rope_scaling")
        required = ["rope_type", "factor", "low_freq_factor", "high_freq_factor", "original_max_position_embeddings"]
        if len(rs) != len(required):
            raise HFError("Llama 3 RoPE requires exactly five canonical fields")
        for k in required:
            if rs.get(k) is None:
                raise HFError(f'missing or null Llama 3 RoPE field "{k}"')
        typ = _field(rs, "rope_type", "str", "")
        fac, low = _field(rs, "factor", "float", 0.0), _field(rs, "low_freq_factor", "float", 0.0)
        high, orig = _field(rs, "high_freq_factor", "float", 0.0), _field(rs, "original_max_position_embeddings",
                                                                         "int", 0)
        f32 = lambda x: float(np.float32(x))  # noqa: E731
        if (mt != "llama" or typ != "llama3" or not all(np.isfinite([fac, low, high])) or fac < 1 or fac > 1e6 or
                low < 1e-6 or high <= low or f32(high) <= f32(low) or high > 1e6 or orig < 1 or orig > 131072 or
                orig > h.max_positions):
            raise HFError("unsupported or invalid Llama 3 RoPE scaling")
        h.rope = dict(factor=fac, low=low, high=high, original=orig)
    arch = _ARCH.get(mt, "")
    act = _field(raw, "hidden_act", "str", "")
    tp = _field(raw, "pretraining_tp", "int", 0)
    if (not arch or h.architectures != [arch] or act != "silu" or _field(raw, "attention_bias", "bool", False) or
            _field(raw, "mlp_bias", "bool", False) or _field(raw, "rope_interleaved", "bool", False) or
            _field(raw, "attention_dropout", "float", 0.0) != 0 or tp not in (0, 1) or
            _field(raw, "use_sliding_window", "bool", False)):
        raise HFError("unsupported HF profile: require Llama, Qwen2 or full-attention Mistral, SiLU, supported "
                      "half-split RoPE and full causal attention")
    lt = _field(raw, "layer_types", "strs", [])
    if lt and len(lt) != h.layers:
        raise HFError("HF layer_types count mismatch")
    if any(x != "full_attention" for x in lt):
        raise HFError("unsupported HF attention layer type")
    if (raw.get("bos_token_id") is None or raw.get("eos_token_id") is None or not 0 <= h.bos < h.vocab or
            not 0 <= h.eos < h.vocab):
        raise HFError("HF profile requires scalar BOS/EOS IDs within vocabulary")
    if context_limit < 0 or context_limit > h.max_positions:
        raise HFError("HF context limit must be within model context")
    h.context = context_limit if context_limit > 0 else min(h.max_positions, 2048)
    # validateShapeLimits (M:100-114) with the HF bounds
    if (h.vocab < BASE_VOCAB or h.vocab > MAX_HF_VOCAB or h.dim < 2 or h.dim > 8192 or h.hidden < 1 or
            h.hidden > 32768 or h.layers < 1 or h.layers > 128 or h.heads < 1 or h.heads > h.dim or h.kv_heads < 1 or
            h.kv_heads > h.heads or h.context < 1 or h.context > 32768):
        raise HFError("invalid model dimensions (see README limits)")
    if h.dim % h.heads or h.heads % h.kv_heads or (h.dim // h.heads) % 2:
        raise HFError("dim must be divisible by heads with an even head dimension; heads must be divisible by "
                      "kv_heads")
    if not np.isfinite(h.theta) or h.theta <= 1 or not np.isfinite(h.eps) or h.eps < 1e-12 or h.eps > 1:
        raise HFError("invalid RoPE theta or RMS epsilon")
    if h.parameter_count() > MAX_HF_PARAMETERS:
        raise HFError(f"HF model exceeds {MAX_HF_PARAMETERS} parameters including biases and output head")
    return h


def read_gpt2_config(raw, context_limit=0):
    """readGPT2Config (M:446-513)."""
    for k, v in raw.items():
        if k not in _GPT2_ALLOWED:
            raise HFError(f'unsupported GPT-2 config field "{k}"')
        if v is None and k not in ("n_inner", "pad_token_id", "summary_activation"):
            raise HFError(f'null GPT-2 config field "{k}"')
    f = lambda k, kind, d: _field(raw, k, kind, d)  # noqa: E731
    h = HFConfig({}, 0)
    h.raw = raw
    h.model_type = "gpt2"
    h.architectures = f("architectures", "strs", [])
    h.vocab = f("vocab_size", "int", 0)
    h.tied = f("tie_word_embeddings", "bool", True)
    h.bos, h.eos = f("bos_token_id", "int", 0), f("eos_token_id", "int", 0)
    dim, hidden = f("n_embd", "int", 0), f("n_inner", "int", 0)
    layers, heads, ctx, nctx = f("n_layer", "int", 0), f("n_head", "int", 0), f("n_positions", "int", 0), \
        f("n_ctx", "int", 0)
    eps, act = f("layer_norm_epsilon", "float", 1e-5), f("activation_function", "str", "gelu_new")
    scale, inverse = f("scale_attn_weights", "bool", True), f("scale_attn_by_inverse_layer_idx", "bool", False)
    upcast, cross = f("reorder_and_upcast_attn", "bool", False), f("add_cross_attention", "bool", False)
    if (h.architectures != ["GPT2LMHeadModel"] or not h.tied or act != "gelu_new" or not scale or inverse or upcast or
            cross or (nctx != 0 and nctx != ctx)):
        raise HFError("unsupported GPT-2 profile: require tied GPT2LMHeadModel, gelu_new and standard scaled causal "
                      "self-attention")
    if hidden == 0:
        hidden = 4 * dim
    h.dim, h.hidden, h.layers, h.heads, h.kv_heads = dim, hidden, layers, heads, heads
    h.max_positions = h.positions = ctx
    h.eps, h.theta = eps, 10000.0
    if "bos_token_id" not in raw or "eos_token_id" not in raw or not 0 <= h.bos < h.vocab or \
            not 0 <= h.eos < h.vocab:
        raise HFError("GPT-2 requires scalar BOS/EOS IDs within vocabulary")
    if context_limit < 0 or context_limit > ctx or ctx > 32768:
        raise HFError("invalid GPT-2 context limit")
    h.context = context_limit if context_limit > 0 else min(ctx, 2048)
    if (h.vocab < BASE_VOCAB or h.vocab > MAX_HF_VOCAB or h.dim < 2 or h.dim > 8192 or h.hidden < 1 or
            h.hidden > 32768 or h.layers < 1 or h.layers > 128 or h.heads < 1 or h.heads > h.dim or
            h.context < 1 or h.context > 32768):
        raise HFError("invalid model dimensions (see README limits)")
    if h.dim % h.heads or (h.dim // h.heads) % 2:
        raise HFError("dim must be divisible by heads with an even head dimension; heads must be divisible by "
                      "kv_heads")
    if not np.isfinite(h.eps) or h.eps < 1e-12 or h.eps > 1:
        raise HFError("invalid RoPE theta or RMS epsilon")
    if h.parameter_count() > MAX_HF_PARAMETERS:
        raise HFError("GPT-2 exceeds HF parameter limit")
    return h


# --------------------------------------------------------------- archive --
def half_float(bits):
    """halfFloat (M:834-847) over an array of IEEE half bit patterns: exact fp32."""
    v = np.asarray(bits, dtype=np.uint16).astype(np.uint32)
    sign = (v & 0x8000) << 16
    exp = (v >> 10) & 31
    frac = v & 1023
    sub = np.ldexp(frac.astype(np.float64), -24).astype(np.float32).view(np.uint32) | sign
    inf_nan = sign | 0x7F800000 | (frac << 13)
    normal = sign | ((exp + 112) << 23) | (frac << 13)
    out = np.where(exp == 0, sub, np.where(exp == 31, inf_nan, normal)).astype(np.uint32)
    return out.view(np.float32)


class _Tensor:
    __slots__ = ("file", "start", "dtype", "shape", "count")

    def __init__(self, file, start, dtype, shape, count):
        self.file, self.start, self.dtype, self.shape, self.count = file, start, dtype, shape, count


class HFArchive:
    """A validated checkpoint directory (hfArchive, M:618-632)."""

    def __init__(self, path, config, tensors, shards):
        self.path, self.config, self.tensors, self.shards = path, config, tensors, shards

    def dtypes(self):
        out = {}
        for t in self.tensors.values():
            out[t.dtype] = out.get(t.dtype, 0) + 1
        return out

    def read_tensor(self, name, threads=None):
        """readTensorValues (M:856-894): the tensor widened to fp32, row-major.
        Large tensors are widened in slices on `threads` host threads (default:
        all cores); the values do not depend on the slicing."""
        t = self.tensors.get(name)
        if t is None:
            raise HFError("HF tensor destination mismatch")
        w = WIDTH[t.dtype]
        mm = np.memmap(t.file, dtype=np.uint8, mode="r", offset=t.start, shape=(t.count * w,))
        src = np.frombuffer(mm, dtype="<f4" if t.dtype == "F32" else "<u2")
        out = np.empty(t.count, dtype=np.float32)
        finite = []

        def widen(lo, hi):
            if t.dtype == "F32":
                out[lo:hi] = src[lo:hi]
            elif t.dtype == "BF16":
                out[lo:hi] = (src[lo:hi].astype(np.uint32) << 16).view(np.float32)
            else:
                out[lo:hi] = half_float(src[lo:hi])
            finite.append(bool(np.isfinite(out[lo:hi]).all()))

        n = threads or os.cpu_count() or 1
        step = 1 << 22
        if n > 1 and t.count > 2 * step:
            from concurrent.futures import ThreadPoolExecutor
            with ThreadPoolExecutor(n) as ex:
                list(ex.map(lambda lo: widen(lo, min(lo + step, t.count)), range(0, t.count, step)))
        else:
            widen(0, t.count)
        del src, mm
        if not all(finite):
            raise HFError(f"non-finite HF weight in {name}")
        return out.reshape(t.shape)

    def params(self):
        """The parameters in the model's order as fp32 arrays: hfProfileSpecs
        order, or loadGPT2's (M:5052-5165) with Conv1D weights transposed to
        [out, in] and c_attn split into q, k, v; GPT-2 legacy causal masks are
        checked (M:5146-5160) and not returned."""
        h = self.config
        if h.model_type != "gpt2":
            for name, _ in h.specs():
                yield self.read_tensor(name)
            return
        d = h.dim
        for name in ("wte.weight", "wpe.weight", "ln_f.weight", "ln_f.bias"):
            yield self.read_tensor(name)
        for i in range(h.layers):
            p = f"h.{i}."
            w = self.read_tensor(p + "attn.c_attn.weight").T
            b = self.read_tensor(p + "attn.c_attn.bias")
            yield self.read_tensor(p + "ln_1.weight")
            yield self.read_tensor(p + "ln_1.bias")
            for part in (w[:d], w[d:2 * d], w[2 * d:], b[:d], b[d:2 * d], b[2 * d:]):
                yield np.ascontiguousarray(part)
            yield np.ascontiguousarray(self.read_tensor(p + "attn.c_proj.weight").T)
            yield self.read_tensor(p + "attn.c_proj.bias")
            yield self.read_tensor(p + "ln_2.weight")
            yield self.read_tensor(p + "ln_2.bias")
            yield np.ascontiguousarray(self.read_tensor(p + "mlp.c_fc.weight").T)
            yield self.read_tensor(p + "mlp.c_fc.bias")
            yield np.ascontiguousarray(self.read_tensor(p + "mlp.c_proj.weight").T)
            yield self.read_tensor(p + "mlp.c_proj.bias")
            mask = p + "attn.bias"
            if mask in self.tensors:
                P = h.positions
                want = np.tril(np.ones((P, P), dtype=np.float32)).reshape(1, 1, P, P)
                if not np.array_equal(self.read_tensor(mask), want):
                    raise HFError("invalid GPT-2 legacy causal mask values")

    def load_into(self, model):
        """Every tensor, in parameter order, through sr_model_load_param_f32 (the
        device quantizer restates readParam, M:857-880).  The next tensor is read
        and widened on a host thread while the current one uploads."""
        from concurrent.futures import ThreadPoolExecutor
        it = self.params()
        with ThreadPoolExecutor(1) as ex:
            pending = ex.submit(next, it, None)
            i = 0
            while True:
                values = pending.result()
                if values is None:
                    break
                pending = ex.submit(next, it, None)
                model.load_param_f32(i, values)
                i += 1


def open_hf_archive(path, context_limit=0):
    """openHFArchiveFormat (M:644-831): config, optional shard index, and every
    shard's header checked before any weight is read."""
    h = read_hf_config(path, context_limit)
    params = h.parameter_count()
    expected = dict(h.specs())
    optional = h.optional()
    aux = sum(int(np.prod(s)) * 4 for s in optional.values())
    index = None
    shards = set()
    ipath = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(ipath):
        raw = read_bounded_json(ipath, MAX_HF_HEADER)
        wm = raw.get("weight_map") if isinstance(raw, dict) else None
        if not isinstance(wm, dict):
            wm = {}
        if len(wm) < len(expected) or len(wm) > len(expected) + len(optional):
            raise HFError("HF shard index tensor count mismatch")
        index = {}
        for name, file in wm.items():
            name = h.canonical(name)
            if ((name not in expected and name not in optional) or name in index or not isinstance(file, str) or
                    not file or
                    os.path.basename(file) != file or "/" in file or "\\" in file or not file.endswith(".safetensors")):
                raise HFError("unsupported HF shard index name/path")
            index[name] = file
            shards.add(file)
    else:
        shards.add("model.safetensors")
    if not 1 <= len(shards) <= 128:
        raise HFError("HF shard count limit")
    tensors = {}
    for name in sorted(shards):
        fpath = os.path.join(path, name)
        if not os.path.isfile(fpath):
            raise HFError(f"open {name}: no such file")
        size = os.path.getsize(fpath)
        if size < 10 or size > params * 4 + aux + MAX_HF_HEADER + 8:
            raise HFError("Safetensors file size/type limit")
        with open(fpath, "rb") as f:
            n = int.from_bytes(f.read(8), "little")
            if n < 2 or n > MAX_HF_HEADER or n > size - 8:
                raise HFError("Safetensors header length limit")
            header = f.read(n)
        if header[:1] != b"{":
            raise HFError("Safetensors header must start with object")
        raw = unique_json(header)
        body = size - 8 - n
        ordered = []
        for key, value in raw.items():
            if key == "__metadata__":
                if not isinstance(value, dict) or not all(isinstance(v, str) for v in value.values()):
                    raise HFError("invalid Safetensors metadata")
                continue
            key = h.canonical(key)
            shape_of = expected.get(key, optional.get(key))
            if shape_of is None or key in tensors or (index is not None and index.get(key) != name):
                raise HFError(f'unexpected or duplicate HF tensor "{key}"')
            if not isinstance(value, dict) or set(value) - {"dtype", "shape", "data_offsets"}:
                raise HFError(f"invalid HF tensor header: {key}")
            shape = value.get("shape")
            if not isinstance(shape, list) or len(shape) != len(shape_of):
                raise HFError(f"HF tensor shape mismatch: {key}")
            if any(not _is_int(a) or a != b for a, b in zip(shape, shape_of)):
                raise HFError(f"HF tensor shape mismatch: {key}")
            count = int(np.prod(shape_of))
            dt = value.get("dtype")
            w = WIDTH.get(dt, 0) if isinstance(dt, str) else 0
            if key in optional and dt != "F32":
                raise HFError("GPT-2 legacy causal masks must be F32")
            off = value.get("data_offsets")
            if (w == 0 or not isinstance(off, list) or len(off) != 2 or not all(_is_int(o) for o in off) or
                    off[0] < 0 or off[1] < off[0] or off[1] > body or off[1] - off[0] != count * w):
                raise HFError(f"invalid HF tensor dtype/extent: {key}")
            tensors[key] = _Tensor(fpath, 8 + n + off[0], dt, tuple(shape_of), count)
            ordered.append(off)
        end = 0
        for lo, hi in sorted(ordered):
            if lo != end:
                raise HFError("Safetensors overlapping or unindexed bytes")
            end = hi
        if end != body:
            raise HFError("Safetensors trailing/unindexed bytes")
    for key in expected:
        if key not in tensors:
            raise HFError(f'missing HF tensor "{key}"')
    return HFArchive(path, h, tensors, sorted(shards))


def load_hf_model(path, weight_format="q8", context_limit=0, page_tokens=32, device=0, tp_rank=0, tp_size=1,
                  nccl_id=None):
    """Open, validate and upload a checkpoint: a device Model (one tensor-parallel
    rank of it when tp_size > 1) holding the archive's weights in `weight_format`."""
    from .step import Model
    a = open_hf_archive(path, context_limit)
    m = Model(a.config.desc(weight_format, page_tokens), device, tp_rank=tp_rank, tp_size=tp_size, nccl_id=nccl_id)
    try:
        a.load_into(m)
    except Exception:
        m.close()
        raise
    return m, a


def _bench(dim=2048, hidden=8192, layers=8, vocab=32000, shards=2, seed=0):
    """Host throughput of the import: a temporary Llama-shaped BF16 checkpoint
    (seeded values, `shards` files with an index) is validated and every tensor
    widened to fp32 in parameter order (the device upload is not included)."""
    import shutil
    import tempfile
    import time
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "vocab_size": vocab, "hidden_size": dim,
           "intermediate_size": hidden, "num_hidden_layers": layers, "num_attention_heads": dim // 64,
           "num_key_value_heads": dim // 256, "max_position_embeddings": 4096, "rope_theta": 5e5,
           "rms_norm_eps": 1e-5, "hidden_act": "silu", "tie_word_embeddings": False, "bos_token_id": 1,
           "eos_token_id": 2}
    h = HFConfig(cfg, 0)
    h.model_type = "llama"
    specs = h.specs()
    rng = np.random.default_rng(seed)
    d = tempfile.mkdtemp(prefix="sr_hf_bench_")
    try:
        with open(os.path.join(d, "config.json"), "w") as f:
            json.dump(cfg, f)
        parts = np.array_split(np.arange(len(specs)), shards)
        wm, total = {}, 0
        for k, idx in enumerate(parts):
            fn = f"model-{k + 1:05d}-of-{shards:05d}.safetensors"
            header, off = {}, 0
            for i in idx:
                name, shape = specs[i]
                n = int(np.prod(shape)) * 2
                header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + n]}
                off += n
                wm[name] = fn
            hb = json.dumps(header).encode()
            with open(os.path.join(d, fn), "wb") as f:
                f.write(len(hb).to_bytes(8, "little"))
                f.write(hb)
                for i in idx:
                    count = int(np.prod(specs[i][1]))
                    f.write((rng.standard_normal(count, dtype=np.float32) * 0.02).view(np.uint32).__rshift__(16)
                            .astype("<u2").tobytes())
            total += off
        with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
            json.dump({"weight_map": wm}, f)
        t0 = time.perf_counter()
        a = open_hf_archive(d)
        t1 = time.perf_counter()
        n = sum(p.size for p in a.params())
        t2 = time.perf_counter()
        print(f"{h.parameter_count():,} parameters, {total / 1e9:.2f} GB BF16 in {shards} shards: "
              f"headers checked in {(t1 - t0) * 1e3:.1f} ms; values read and widened at {total / (t2 - t1) / 1e9:.2f} "
              f"GB/s of checkpoint ({n / (t2 - t1) / 1e6:.0f} M values/s), {os.cpu_count()} host threads")
    finally:
        shutil.rmtree(d)


if __name__ == "__main__":
    import sys
    if "--bench" in sys.argv:
        _bench()
