"""ctypes declarations for libsrstep.so (include/srstep.h).

The library is loaded from this package directory; there is no fallback: if it
is missing or fails to load, importing the step API raises.
"""

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsrstep.so")

SR_OK, SR_EINVAL, SR_ECANCELED, SR_ENOMEM, SR_ETIMEOUT, SR_EDEVICE, SR_EUNSUPPORTED = range(7)
SR_FMT_F32, SR_FMT_Q8, SR_FMT_Q4, SR_FMT_Q4_MIXED = range(4)
SR_PARAM_F32, SR_PARAM_Q8, SR_PARAM_Q4 = range(3)
SR_MODE_EXACT, SR_MODE_FAST = 0, 1
SR_TP_PEER_HANDLE_BYTES = 64
SR_TEXT_HF, SR_TEXT_CLEANUP, SR_TEXT_MISTRAL = 1, 2, 4
SR_ARCH_LLAMA, SR_ARCH_GPT2 = 0, 1
SR_PEER_BARRIER, SR_PEER_LL = 0, 1
FORMATS = {"f32": SR_FMT_F32, "q8": SR_FMT_Q8, "q4": SR_FMT_Q4, "q4-mixed": SR_FMT_Q4_MIXED}

# Every symbol include/srstep.h declares (checked by tests/test_abi.py).
EXPORTED = [
    "sr_last_error", "sr_version", "sr_model_create", "sr_model_destroy", "sr_model_param_count",
    "sr_model_param_info", "sr_model_load_param", "sr_model_load_param_f32", "sr_model_read_param",
    "sr_model_init_synthetic", "sr_model_set_mode", "sr_kvpool_create", "sr_kvpool_destroy", "sr_kvpool_read_row",
    "sr_kvpool_fill_synthetic", "sr_step", "sr_step_logits", "sr_sample", "sr_step_sample", "sr_engine_create",
    "sr_engine_destroy", "sr_engine_submit", "sr_engine_tick", "sr_engine_poll", "sr_engine_stats_get",
    "sr_engine_last_schedule", "sr_engine_session_pages", "sr_profile_set", "sr_profile_read", "sr_model_stream",
    "sr_step_noalloc", "sr_model_create_tp", "sr_tp_unique_id", "sr_tp_shard", "sr_engine_latency",
    "sr_kvpool_copy_rows", "sr_engine_clear_prefix", "sr_tp_peer_handle", "sr_tp_peer_open",
    "sr_text_decoder_create", "sr_text_decoder_destroy", "sr_text_decoder_push", "sr_text_decoder_push_token",
    "sr_tp_peer_set_protocol", "sr_engine_set_pieces", "sr_engine_poll_token", "sr_sample_logits",
    "sr_linear", "sr_model_set_code_cache", "sr_model_code_cache", "sr_model_set_split",
]
PROF_CLASSES = ["meta", "embed", "norm", "linear", "rope_kv", "attention", "swiglu", "head", "sample"]


class ModelDesc(C.Structure):
    _fields_ = [("vocab", C.c_int32), ("dim", C.c_int32), ("hidden", C.c_int32), ("layers", C.c_int32),
                ("heads", C.c_int32), ("kv_heads", C.c_int32), ("context", C.c_int32),
                ("rope_theta", C.c_double), ("norm_eps", C.c_double), ("tied", C.c_int32),
                ("qkv_bias", C.c_int32), ("weight_format", C.c_int32), ("page_tokens", C.c_int32),
                ("rope_scaling", C.c_int32), ("rope_factor", C.c_double), ("rope_low_freq_factor", C.c_double),
                ("rope_high_freq_factor", C.c_double), ("rope_original_max_positions", C.c_int32),
                ("arch", C.c_int32), ("positions", C.c_int32)]


class ParamInfo(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("format", C.c_int32), ("reserved", C.c_int32),
                ("value_bytes", C.c_int64), ("scale_count", C.c_int64)]


class Batch(C.Structure):
    _fields_ = [("n_sessions", C.c_int32), ("pos", C.c_void_p), ("token_offsets", C.c_void_p),
                ("tokens", C.c_void_p), ("page_offsets", C.c_void_p), ("page_ids", C.c_void_p),
                ("want_logits", C.c_void_p)]


class Sampling(C.Structure):
    _fields_ = [("temperature", C.c_double), ("top_k", C.c_int32), ("reserved", C.c_int32),
                ("top_p", C.c_double), ("repeat_penalty", C.c_double)]


class EngineConfig(C.Structure):
    _fields_ = [("max_batch", C.c_int32), ("token_budget", C.c_int32), ("prefill_chunk", C.c_int32),
                ("mixed_prefill_chunk", C.c_int32), ("cache_bytes", C.c_int64), ("eos_id", C.c_int32),
                ("blocked_id", C.c_int32), ("prefix_cache_bytes", C.c_int64), ("prefix_cache_tail", C.c_int32),
                ("reserved", C.c_int32)]


class Request(C.Structure):
    _fields_ = [("ids", C.c_void_p), ("n_ids", C.c_int32), ("max_tokens", C.c_int32), ("sampling", Sampling),
                ("seed", C.c_uint64)]


class EngineStats(C.Structure):
    _fields_ = [(k, C.c_int64) for k in ("submitted", "completed", "rejected", "failed", "active", "queued",
                                          "input_tokens", "generated_tokens", "ticks", "peak_tick_tokens",
                                          "pool_limit", "pool_reserved", "pool_allocated", "prefix_hits",
                                          "prefix_tokens", "prefix_bytes")]


class SRError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None


def lib():
    """Load libsrstep.so from the package directory (raises if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m sr_go_tranformer_b200.build`")
    L = C.CDLL(LIB_PATH)
    P, I32, I64, U64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint64
    sig = {
        "sr_last_error": (C.c_char_p, []),
        "sr_version": (C.c_char_p, []),
        "sr_model_create": (C.c_int, [C.POINTER(ModelDesc), C.c_int, C.POINTER(P)]),
        "sr_model_destroy": (C.c_int, [P]),
        "sr_model_param_count": (C.c_int, [P, C.POINTER(I32)]),
        "sr_model_param_info": (C.c_int, [P, I32, C.POINTER(ParamInfo)]),
        "sr_model_load_param": (C.c_int, [P, I32, P, C.c_size_t, P, C.c_size_t]),
        "sr_model_load_param_f32": (C.c_int, [P, I32, P, C.c_size_t]),
        "sr_model_read_param": (C.c_int, [P, I32, P, C.c_size_t, P, C.c_size_t]),
        "sr_model_init_synthetic": (C.c_int, [P, U64, C.c_double]),
        "sr_model_set_mode": (C.c_int, [P, I32]),
        "sr_kvpool_create": (C.c_int, [P, I64, C.POINTER(P)]),
        "sr_kvpool_destroy": (C.c_int, [P]),
        "sr_kvpool_read_row": (C.c_int, [P, I64, I32, I32, P, P]),
        "sr_kvpool_fill_synthetic": (C.c_int, [P, U64, C.c_float]),
        "sr_kvpool_copy_rows": (C.c_int, [P, I64, I64, I32]),
        "sr_engine_clear_prefix": (C.c_int, [P]),
        "sr_step": (C.c_int, [P, P, C.POINTER(Batch), P, P]),
        "sr_step_logits": (C.c_int, [P, C.POINTER(P)]),
        "sr_step_noalloc": (C.c_int, [P, P, C.POINTER(Batch), P]),
        "sr_model_create_tp": (C.c_int, [C.POINTER(ModelDesc), C.c_int, I32, I32, P, C.POINTER(P)]),
        "sr_tp_unique_id": (C.c_int, [P]),
        "sr_tp_shard": (C.c_int, [C.POINTER(ModelDesc), I32, I32, I32, P]),
        "sr_tp_peer_handle": (C.c_int, [P, P]),
        "sr_tp_peer_open": (C.c_int, [P, P]),
        "sr_tp_peer_set_protocol": (C.c_int, [P, I32]),
        "sr_engine_set_pieces": (C.c_int, [P, P, P, I32, I32, P]),
        "sr_engine_poll_token": (C.c_int, [P, C.POINTER(I64), C.POINTER(I32), P, I32, C.POINTER(I32),
                                           C.POINTER(I32)]),
        "sr_text_decoder_create": (C.c_int, [I32, P, I32, C.POINTER(P)]),
        "sr_text_decoder_destroy": (C.c_int, [P]),
        "sr_text_decoder_push": (C.c_int, [P, P, I64, I32, P, I64, C.POINTER(I64), C.POINTER(I64)]),
        "sr_text_decoder_push_token": (C.c_int, [P, I32, P, I64, I32, P, I64, C.POINTER(I64), C.POINTER(I64)]),
        "sr_sample": (C.c_int, [P, I32, P, P, P, P, I32, P]),
        "sr_sample_logits": (C.c_int, [P, I32, I32, P, P, P, P, P, I32, P]),
        "sr_linear": (C.c_int, [P, I32, I32, P, P]),
        "sr_model_set_code_cache": (C.c_int, [P, I32]),
        "sr_model_code_cache": (C.c_int, [P, C.POINTER(I32)]),
        "sr_model_set_split": (C.c_int, [P, I32]),
        "sr_step_sample": (C.c_int, [P, P, C.POINTER(Batch), P, P, P, P, I32, P]),
        "sr_engine_create": (C.c_int, [P, C.POINTER(EngineConfig), C.POINTER(P)]),
        "sr_engine_destroy": (C.c_int, [P]),
        "sr_engine_submit": (C.c_int, [P, C.POINTER(Request), C.POINTER(I64)]),
        "sr_engine_tick": (C.c_int, [P, C.POINTER(I32)]),
        "sr_engine_poll": (C.c_int, [P, C.POINTER(I64), P, I32, C.POINTER(I32), C.POINTER(I32)]),
        "sr_engine_stats_get": (C.c_int, [P, C.POINTER(EngineStats)]),
        "sr_engine_latency": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(I64),
                                        C.POINTER(I64)]),
        "sr_engine_last_schedule": (C.c_int, [P, P, I32, C.POINTER(I32)]),
        "sr_engine_session_pages": (C.c_int, [P, I32, P, I32, C.POINTER(I32)]),
        "sr_profile_set": (C.c_int, [P, C.c_uint32]),
        "sr_profile_read": (C.c_int, [P, P, P, C.POINTER(C.c_double), C.POINTER(I64), C.POINTER(I64), I32]),
        "sr_model_stream": (C.c_int, [P, C.POINTER(P)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(rc):
    if rc != SR_OK:
        raise SRError(rc, lib().sr_last_error().decode())
    return rc
