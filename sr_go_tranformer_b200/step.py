"""Host-side mirror of the reference's step API over libsrstep.so.

Names and argument meaning follow cmd/monolith/monolith.go ("M:line"):
`Model.prefill_selected(caches, chunks, want_logits)` is prefillSelected
(M:6245), `prefill_batch` / `decode_batch` / `step` are PrefillBatch /
DecodeBatch / Step (M:6198-6216, 6457), `KVCache` (M:5954) holds the committed
position and its page ids, and `PagePool` is the engine's LIFO pagePool
(M:5849-5866) whose pages live in one device pool.  Errors raise SRError (the
reference returns a Go error); invalid input mutates nothing.
"""

import ctypes as C
import json

import numpy as np

from . import _abi as A


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def desc_from_hf(hf, weight_format="f32", page_tokens=32, context=None):
    """sr_model_desc from an HF config.json dict (readHFConfig, M:253-385;
    readGPT2Config, M:446-513, for model_type gpt2)."""
    d = A.ModelDesc()
    if hf.get("model_type") == "gpt2":
        d.vocab, d.dim, d.layers = hf["vocab_size"], hf["n_embd"], hf["n_layer"]
        d.hidden = hf.get("n_inner") or 4 * d.dim
        d.heads = d.kv_heads = hf["n_head"]
        d.positions = hf["n_positions"]
        d.context = context or min(d.positions, 2048)
        d.rope_theta, d.norm_eps = 10000.0, float(hf.get("layer_norm_epsilon", 1e-5))
        d.tied, d.qkv_bias, d.arch = 1, 0, A.SR_ARCH_GPT2
        d.weight_format = A.FORMATS[weight_format]
        d.page_tokens = page_tokens
        return d
    d.vocab = hf["vocab_size"]
    d.dim = hf["hidden_size"]
    d.hidden = hf["intermediate_size"]
    d.layers = hf["num_hidden_layers"]
    d.heads = hf["num_attention_heads"]
    d.kv_heads = hf.get("num_key_value_heads", d.heads)
    d.context = context or hf.get("max_position_embeddings", 2048)
    d.rope_theta = float(hf.get("rope_theta", 10000.0))
    d.norm_eps = float(hf.get("rms_norm_eps", 1e-6))
    d.tied = 1 if hf.get("tie_word_embeddings", False) else 0
    d.qkv_bias = 1 if hf.get("model_type") == "qwen2" else 0
    d.weight_format = A.FORMATS[weight_format]
    d.page_tokens = page_tokens
    rs = hf.get("rope_scaling")
    if rs:
        d.rope_scaling = 1
        d.rope_factor = float(rs["factor"])
        d.rope_low_freq_factor = float(rs["low_freq_factor"])
        d.rope_high_freq_factor = float(rs["high_freq_factor"])
        d.rope_original_max_positions = int(rs["original_max_position_embeddings"])
    return d


def make_desc(vocab, dim, hidden, layers, heads, kv_heads, context, rope_theta=1e4, norm_eps=1e-5, tied=True,
              qkv_bias=False, weight_format="f32", page_tokens=32):
    d = A.ModelDesc()
    d.vocab, d.dim, d.hidden, d.layers, d.heads, d.kv_heads, d.context = (vocab, dim, hidden, layers, heads,
                                                                          kv_heads, context)
    d.rope_theta, d.norm_eps = float(rope_theta), float(norm_eps)
    d.tied, d.qkv_bias = int(tied), int(qkv_bias)
    d.weight_format, d.page_tokens = A.FORMATS[weight_format], page_tokens
    return d


def tp_unique_id():
    """128-byte NCCL id (rank 0) for Model(..., tp_rank, tp_size, nccl_id)."""
    buf = (C.c_char * 128)()
    A.check(A.lib().sr_tp_unique_id(buf))
    return bytes(buf)


def tp_shard(desc, rank, size, index):
    """(row0, rows, col0, cols) of parameter `index` held by rank `rank` of `size`."""
    out = np.zeros(4, dtype=np.int32)
    A.check(A.lib().sr_tp_shard(C.byref(desc), rank, size, index, _p(out)))
    return tuple(int(x) for x in out)


class Model:
    """A device model (weights, RoPE tables, workspace) on one GPU, or one
    tensor-parallel rank of it (tp_size > 1, nccl_id from tp_unique_id)."""

    def __init__(self, desc, device=0, tp_rank=0, tp_size=1, nccl_id=None):
        self.desc = desc
        self.tp_rank, self.tp_size = tp_rank, tp_size
        h = C.c_void_p()
        if tp_size > 1:
            idbuf = C.create_string_buffer(bytes(nccl_id), 128)
            A.check(A.lib().sr_model_create_tp(C.byref(desc), device, tp_rank, tp_size, idbuf, C.byref(h)))
        else:
            A.check(A.lib().sr_model_create(C.byref(desc), device, C.byref(h)))
        self.h = h
        n = C.c_int32()
        A.check(A.lib().sr_model_param_count(self.h, C.byref(n)))
        self.nparams = n.value
        self.vocab = desc.vocab
        self._direct_pool = None

    def close(self):
        if getattr(self, "h", None):
            if self._direct_pool is not None:
                self._direct_pool.close()
            A.lib().sr_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tp_peer_handle(self):
        """This rank's CUDA IPC handle of its all-reduce buffers (bytes)."""
        buf = C.create_string_buffer(A.SR_TP_PEER_HANDLE_BYTES)
        A.check(A.lib().sr_tp_peer_handle(self.h, buf))
        return buf.raw

    def tp_peer_open(self, handles):
        """Map every rank's buffers (handles in rank order) and all-reduce over
        NVLink peer memory from now on instead of NCCL."""
        blob = b"".join(bytes(h) for h in handles)
        assert len(blob) == A.SR_TP_PEER_HANDLE_BYTES * self.tp_size
        A.check(A.lib().sr_tp_peer_open(self.h, C.create_string_buffer(blob, len(blob))))

    def tp_peer_set_protocol(self, protocol):
        """"barrier" (two kernels with flag barriers) or "ll" (one kernel, flags
        inside every 16-byte line); after tp_peer_open, the same on every rank."""
        A.check(A.lib().sr_tp_peer_set_protocol(self.h, {"barrier": A.SR_PEER_BARRIER, "ll": A.SR_PEER_LL}[protocol]))

    @property
    def page_tokens(self):
        return self.desc.page_tokens

    @property
    def kv_dim(self):
        """KV width held on this device (this rank's KV heads: the rows of its
        layer-0 k_proj shard)."""
        if self.tp_size == 1:
            return self.desc.dim // self.desc.heads * self.desc.kv_heads
        return tp_shard(self.desc, self.tp_rank, self.tp_size, 3)[1]

    @property
    def page_elements(self):
        return 2 * self.desc.page_tokens * self.kv_dim * self.desc.layers

    def set_mode(self, mode):
        A.check(A.lib().sr_model_set_mode(self.h, {"exact": A.SR_MODE_EXACT, "fast": A.SR_MODE_FAST}.get(mode, mode)))

    def set_code_cache(self, enabled):
        """Fast mode: keep the fp16 code cache (True, default) or read the
        reference codes as stored (False); see sr_model_set_code_cache."""
        A.check(A.lib().sr_model_set_code_cache(self.h, 1 if enabled else 0))

    def code_cache(self):
        v = C.c_int32()
        A.check(A.lib().sr_model_code_cache(self.h, C.byref(v)))
        return bool(v.value)

    def set_split(self, enabled):
        """Fast-mode steps of enough rows run as two halves on two SM
        partitions (True) or whole (False, the default); see sr_model_set_split."""
        A.check(A.lib().sr_model_set_split(self.h, 1 if enabled else 0))

    def param_info(self, i):
        info = A.ParamInfo()
        A.check(A.lib().sr_model_param_info(self.h, i, C.byref(info)))
        return info

    def load_param(self, i, values, scales=None):
        values = np.ascontiguousarray(values)
        sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
        A.check(A.lib().sr_model_load_param(self.h, i, _p(values), values.nbytes, _p(sc), 0 if sc is None else sc.size))

    def load_param_f32(self, i, values):
        v = np.ascontiguousarray(values, dtype=np.float32)
        A.check(A.lib().sr_model_load_param_f32(self.h, i, _p(v), v.size))

    def read_param(self, i):
        info = self.param_info(i)
        if info.format == A.SR_PARAM_F32:
            vals = np.zeros(info.rows * info.cols, dtype=np.float32)
            A.check(A.lib().sr_model_read_param(self.h, i, _p(vals), vals.nbytes, None, 0))
            return vals, None
        vals = np.zeros(info.value_bytes, dtype=np.int8 if info.format == A.SR_PARAM_Q8 else np.uint8)
        sc = np.zeros(info.scale_count, dtype=np.float32)
        A.check(A.lib().sr_model_read_param(self.h, i, _p(vals), vals.nbytes, _p(sc), sc.size))
        return vals, sc

    def linear(self, index, x):
        """y = x W^T for matrix parameter `index` in the model's mode
        (linearIntoWithExecutor, M:3942); x [rows, in] -> y [rows, out]."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        info = self.param_info(index)
        if x.ndim != 2 or x.shape[1] != info.cols:
            raise A.SRError(A.SR_EINVAL, "x must be [rows, in]")
        y = np.zeros((x.shape[0], info.rows), dtype=np.float32)
        A.check(A.lib().sr_linear(self.h, index, x.shape[0], _p(x), _p(y)))
        return y

    def init_synthetic(self, seed, scale=0.02):
        A.check(A.lib().sr_model_init_synthetic(self.h, seed, scale))

    def new_cache(self, pool=None):
        """Model.NewCache (M:6000); without a pool the model's direct pool is used."""
        if pool is None:
            if self._direct_pool is None:
                pages = (self.desc.context + self.page_tokens - 1) // self.page_tokens
                self._direct_pool = PagePool(self, pages * 4)
            pool = self._direct_pool
        return KVCache(self, pool)

    # -------------------------------------------------------------- the step --
    def prefill_selected(self, caches, chunks, want_logits=None, logits=True, cancel=None):
        """prefillSelected (M:6245-6456): validate, acquire pages lazily (LIFO),
        run the device step, commit Pos += len(chunk) on success."""
        S = len(caches)
        if S < 1 or S > 256 or len(chunks) != S:
            raise A.SRError(A.SR_EINVAL, "invalid prefill batch (1..256 sessions)")
        if want_logits is not None and len(want_logits) != S:
            raise A.SRError(A.SR_EINVAL, "logit selection must match sessions")
        seen = set()
        n = 0
        need = {}
        for c, ch in zip(caches, chunks):
            if c is None or c.model is not self or c.released or id(c) in seen:
                raise A.SRError(A.SR_EINVAL, "foreign, stale, released, or duplicate KV cache")
            seen.add(id(c))
            if len(ch) < 1 or len(ch) > 1024 - n:
                raise A.SRError(A.SR_EINVAL, "prefill requires nonempty chunks totaling at most 1024 tokens")
            if c.pos < 0 or c.pos > self.desc.context or len(ch) > self.desc.context - c.pos:
                raise A.SRError(A.SR_EINVAL, "KV cache context exhausted or invalid position")
            for t in ch:
                if t < 0 or t >= self.vocab:
                    raise A.SRError(A.SR_EINVAL, "token outside vocabulary")
            pages = (c.pos + len(ch) + self.page_tokens - 1) // self.page_tokens
            need[c.pool] = need.get(c.pool, 0) + max(0, pages - len(c.pages))
            n += len(ch)
        for pool, k in need.items():
            if k > pool.available():
                raise A.SRError(A.SR_EINVAL, "insufficient KV page reservation")
        pools = {id(c.pool) for c in caches}
        if len(pools) != 1:
            raise A.SRError(A.SR_EINVAL, "all caches of one step must share a page pool")
        pool = caches[0].pool
        for c, ch in zip(caches, chunks):  # ensurePages after validation (M:6362-6364)
            c.ensure_pages(c.pos + len(ch))
        pos = np.array([c.pos for c in caches], dtype=np.int32)
        toff = np.zeros(S + 1, dtype=np.int32)
        toff[1:] = np.cumsum([len(ch) for ch in chunks])
        tokens = np.concatenate([np.asarray(ch, dtype=np.int32) for ch in chunks]).astype(np.int32)
        poff = np.zeros(S + 1, dtype=np.int32)
        poff[1:] = np.cumsum([len(c.pages) for c in caches])
        pids = np.concatenate([np.asarray(c.pages, dtype=np.int32) for c in caches]).astype(np.int32)
        want = None if want_logits is None else np.asarray([1 if w else 0 for w in want_logits], dtype=np.uint8)
        b = A.Batch(S, _p(pos).value, _p(toff).value, _p(tokens).value, _p(poff).value, _p(pids).value,
                    None if want is None else _p(want).value)
        out = np.zeros((S, self.vocab), dtype=np.float32) if logits else None
        cflag = None
        if cancel is not None:
            cflag = cancel
        A.check(A.lib().sr_step(self.h, pool.h, C.byref(b), _p(out), None if cflag is None else C.byref(cflag)))
        for c, ch in zip(caches, chunks):  # commit (M:6452-6454)
            c.pos += len(ch)
        return out

    def prefill_batch(self, caches, chunks):
        return self.prefill_selected(caches, chunks, None)

    def decode_batch(self, caches, tokens):
        if len(tokens) != len(caches) or len(caches) < 1 or len(caches) > 256:
            raise A.SRError(A.SR_EINVAL, "invalid decode batch (1..256)")
        return self.prefill_selected(caches, [[t] for t in tokens])

    def step(self, cache, token):
        return self.decode_batch([cache], [token])[0]

    @staticmethod
    def _sample_args(settings, histories, rng_states):
        S = len(settings)
        arr = (A.Sampling * S)()
        for i, (t, k, p, pen) in enumerate(settings):
            arr[i] = A.Sampling(t, k, 0, p, pen)
        hoff = np.zeros(S + 1, dtype=np.int32)
        hoff[1:] = np.cumsum([len(h) for h in histories])
        hist = np.concatenate([np.asarray(h, dtype=np.int32) for h in histories] + [np.zeros(1, np.int32)])
        rng = np.asarray(rng_states, dtype=np.uint64).copy()
        ids = np.full(S, -1, dtype=np.int32)
        return S, arr, hoff, hist, rng, ids

    def sample(self, settings, histories, rng_states, blocked=-1):
        """Device sampleWithBlocked over the last step's selected rows.
        settings: list of (temperature, top_k, top_p, penalty); returns ids, rng."""
        S, arr, hoff, hist, rng, ids = self._sample_args(settings, histories, rng_states)
        A.check(A.lib().sr_sample(self.h, S, C.cast(arr, C.c_void_p), _p(hoff), _p(hist), _p(rng), blocked, _p(ids)))
        return ids, rng

    def sample_logits(self, logits, settings, histories, rng_states, blocked=-1):
        """Device sampleWithBlocked(logits, history, s, rng, blocked) over the
        caller's logits [sessions, vocab] (M:7320); returns ids, rng."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        S, arr, hoff, hist, rng, ids = self._sample_args(settings, histories, rng_states)
        if lg.ndim != 2 or lg.shape[0] != S:
            raise A.SRError(A.SR_EINVAL, "logits must be [sessions, vocab]")
        A.check(A.lib().sr_sample_logits(self.h, S, lg.shape[1], _p(lg), C.cast(arr, C.c_void_p), _p(hoff),
                                          _p(hist), _p(rng), blocked, _p(ids)))
        return ids, rng


class PagePool:
    """pagePool (M:5849-5866) whose page ids index one device KV pool."""

    def __init__(self, model, limit):
        self.model = model
        self.limit = int(limit)
        self.reserved = 0
        self.allocated = 0
        self.free = []
        h = C.c_void_p()
        A.check(A.lib().sr_kvpool_create(model.h, self.limit, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            A.lib().sr_kvpool_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def available(self):
        return len(self.free) + self.limit - self.allocated

    def acquire(self):
        if self.free:
            return self.free.pop()
        if self.allocated >= self.limit:
            raise RuntimeError("KV reservation invariant violated")
        self.allocated += 1
        return self.allocated - 1

    def read_row(self, page, layer, slot):
        kd = self.model.kv_dim
        k = np.zeros(kd, dtype=np.float32)
        v = np.zeros(kd, dtype=np.float32)
        A.check(A.lib().sr_kvpool_read_row(self.h, page, layer, slot, _p(k), _p(v)))
        return k, v

    def fill_synthetic(self, seed, scale=1.0):
        A.check(A.lib().sr_kvpool_fill_synthetic(self.h, seed, scale))

    def copy_rows(self, dst, src, rows):
        """copyKVPrefixRows (M:5907-5914): the first `rows` slots of every layer's K
        and V planes of page src into page dst, on the model's stream."""
        A.check(A.lib().sr_kvpool_copy_rows(self.h, int(dst), int(src), int(rows)))


class KVCache:
    """KVCache (M:5954-6062): committed position and page ids."""

    def __init__(self, model, pool):
        self.model = model
        self.pool = pool
        self.pos = 0
        self.pages = []
        self.released = False

    def ensure_pages(self, end):
        needed = (end + self.model.page_tokens - 1) // self.model.page_tokens
        while len(self.pages) < needed:
            self.pages.append(self.pool.acquire())

    def row(self, layer, pos):
        """K and V rows of (layer, pos) (KVCache.row, M:6038-6043)."""
        pt = self.model.page_tokens
        return self.pool.read_row(self.pages[pos // pt], layer, pos % pt)

    def close(self):
        if self.released:
            return
        self.pool.free.extend(self.pages)
        self.pages = []
        self.released = True


def load_hf_fixture(path, weight_format="f32", page_tokens=32, context=None, device=0):
    """Build a device Model from a golden .npz (HF config + fp32 weights in
    hfProfileSpecs order), quantising on the device like readParam."""
    z = np.load(path)
    hf = json.loads(str(z["config"]))
    m = Model(desc_from_hf(hf, weight_format, page_tokens, context), device)
    for i in range(m.nparams):
        m.load_param_f32(i, z[f"param_{i}"])
    return m, z, hf
