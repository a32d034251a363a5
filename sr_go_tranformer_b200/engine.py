"""Python handle on the C++ engine restatement (sr_engine_*, include/srstep.h).

Mirrors the reference Engine (cmd/monolith/monolith.go:7629-8476): submit
requests of token ids, tick the actor loop, poll finished completions.
"""

import ctypes as C

import numpy as np

from . import _abi as A


class Engine:
    REASONS = {0: "length", 1: "eos", 2: "error", 3: "busy"}

    def __init__(self, model, max_batch, token_budget=0, prefill_chunk=0, mixed_prefill_chunk=0, cache_bytes=0,
                 eos_id=-1, blocked_id=-1, prefix_cache_bytes=0, prefix_cache_tail=False):
        """prefix_cache_bytes / prefix_cache_tail: EngineConfig.PrefixCacheBytes /
        PrefixCacheTail (M:7639-7640), the one-entry prefix snapshot's allowance
        carved out of cache_bytes and sub-page reuse."""
        self.model = model
        cfg = A.EngineConfig(max_batch, token_budget, prefill_chunk, mixed_prefill_chunk, int(cache_bytes), eos_id,
                             blocked_id, int(prefix_cache_bytes), int(bool(prefix_cache_tail)), 0)
        h = C.c_void_p()
        A.check(A.lib().sr_engine_create(model.h, C.byref(cfg), C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            A.lib().sr_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, ids, max_tokens, temperature=0.0, top_k=0, top_p=1.0, repeat_penalty=1.0, seed=1):
        arr = np.ascontiguousarray(ids, dtype=np.int32)
        req = A.Request(arr.ctypes.data_as(C.c_void_p), arr.size, max_tokens,
                        A.Sampling(temperature, top_k, 0, top_p, repeat_penalty), seed)
        rid = C.c_int64()
        A.check(A.lib().sr_engine_submit(self.h, C.byref(req), C.byref(rid)))
        return rid.value

    def tick(self):
        rows = C.c_int32()
        A.check(A.lib().sr_engine_tick(self.h, C.byref(rows)))
        return rows.value

    def poll(self, cap=1 << 16):
        out = np.zeros(cap, dtype=np.int32)
        rid, n, reason = C.c_int64(), C.c_int32(), C.c_int32()
        A.check(A.lib().sr_engine_poll(self.h, C.byref(rid), out.ctypes.data_as(C.c_void_p), cap, C.byref(n),
                                       C.byref(reason)))
        if rid.value < 0:
            return None
        return rid.value, out[:n.value].tolist(), self.REASONS[reason.value]

    def stats(self):
        s = A.EngineStats()
        A.check(A.lib().sr_engine_stats_get(self.h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in A.EngineStats._fields_}

    def latency(self):
        """p50 time to first token and p50 inter-token gap (ms) so far, with sample counts."""
        t, g, nt, ng = C.c_double(), C.c_double(), C.c_int64(), C.c_int64()
        A.check(A.lib().sr_engine_latency(self.h, C.byref(t), C.byref(g), C.byref(nt), C.byref(ng)))
        return {"ttft_p50_ms": t.value, "itl_p50_ms": g.value, "first_tokens": nt.value, "gaps": ng.value}

    def set_pieces(self, pieces, hf=False, cleanup=False, mistral=False, fallback=None):
        """Token events with text (TokenEvent, M:8451-8462): pieces[i] is the bytes
        of token i; the flags are the decoder's (newTextDecoder).  Call while idle."""
        blob = b"".join(bytes(p) for p in pieces)
        off = np.zeros(len(pieces) + 1, dtype=np.int64)
        off[1:] = np.cumsum([len(p) for p in pieces])
        flags = (A.SR_TEXT_HF if hf else 0) | (A.SR_TEXT_CLEANUP if cleanup else 0) | \
            (A.SR_TEXT_MISTRAL if mistral else 0)
        fb = None if fallback is None else np.ascontiguousarray(fallback, dtype=np.uint8)
        self._pieces = (blob, off, fb)  # kept alive for the call
        A.check(A.lib().sr_engine_set_pieces(self.h, C.create_string_buffer(blob, max(len(blob), 1)),
                                             off.ctypes.data_as(C.c_void_p), len(pieces), flags,
                                             None if fb is None else fb.ctypes.data_as(C.c_void_p)))

    def poll_token(self):
        """(request id, token id, text, final) of the oldest token event, or None."""
        rid, tid, n, fin = C.c_int64(), C.c_int32(), C.c_int32(), C.c_int32()
        cap = 4096
        while True:
            buf = C.create_string_buffer(cap)
            rc = A.lib().sr_engine_poll_token(self.h, C.byref(rid), C.byref(tid), buf, cap, C.byref(n), C.byref(fin))
            if rc == A.SR_EINVAL and n.value > cap:
                cap = n.value
                continue
            A.check(rc)
            break
        if rid.value < 0:
            return None
        return rid.value, tid.value, buf.raw[:n.value].decode("utf-8"), bool(fin.value)

    def clear_prefix(self):
        """Drop the prefix snapshot (clearPrefix, M:8236-8241); applied once the engine is idle."""
        A.check(A.lib().sr_engine_clear_prefix(self.h))

    def last_schedule(self, cap=256):
        out = np.zeros(cap, dtype=np.int32)
        n = C.c_int32()
        A.check(A.lib().sr_engine_last_schedule(self.h, out.ctypes.data_as(C.c_void_p), cap, C.byref(n)))
        return out[:n.value].tolist()

    def session_pages(self, i, cap=1 << 16):
        out = np.zeros(cap, dtype=np.int32)
        n = C.c_int32()
        A.check(A.lib().sr_engine_session_pages(self.h, i, out.ctypes.data_as(C.c_void_p), cap, C.byref(n)))
        return out[:n.value].tolist()

    def run_to_completion(self, max_ticks=1 << 20):
        done = {}
        for _ in range(max_ticks):
            rows = self.tick()
            while True:
                f = self.poll()
                if f is None:
                    break
                done[f[0]] = (f[1], f[2])
            st = self.stats()
            if rows == 0 and st["active"] == 0 and st["queued"] == 0:
                break
        return done
