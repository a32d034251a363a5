"""Streaming detokenization over libsrstep.so (sr_text_decoder_*, host only).

TextDecoder mirrors the reference's incrementalText (cmd/monolith/monolith.go:
7649-7780) and the Mistral PushToken (M:2132-2161): push each token's piece
and get back the text that is final so far.
"""

import ctypes as C

import numpy as np

from . import _abi as A


class TextDecoder:
    def __init__(self, hf=False, cleanup=False, mistral=False, fallback=None):
        """hf: ByteLevel lossy UTF-8 (HF tokenizers); cleanup: Transformers'
        cleanup cascade; mistral: byte-fallback runs and the leading space, with
        `fallback` the per-id byte-fallback flags of the vocabulary."""
        flags = (A.SR_TEXT_HF if hf else 0) | (A.SR_TEXT_CLEANUP if cleanup else 0) | \
            (A.SR_TEXT_MISTRAL if mistral else 0)
        fb = None if fallback is None else np.ascontiguousarray(fallback, dtype=np.uint8)
        h = C.c_void_p()
        A.check(A.lib().sr_text_decoder_create(flags, None if fb is None else fb.ctypes.data_as(C.c_void_p),
                                               0 if fb is None else fb.size, C.byref(h)))
        self.h = h
        self._fb = fb

    def close(self):
        if getattr(self, "h", None):
            A.lib().sr_text_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _call(self, fn, args, n):
        cap = 3 * n + 256
        out = C.create_string_buffer(cap)
        got, queued = C.c_int64(), C.c_int64()
        A.check(fn(*args, out, cap, C.byref(got), C.byref(queued)))
        text = out.raw[:got.value]
        while queued.value:
            more = C.create_string_buffer(queued.value + 4)
            A.check(A.lib().sr_text_decoder_push(self.h, None, 0, 0, more, queued.value + 4, C.byref(got),
                                                 C.byref(queued)))
            text += more.raw[:got.value]
        return text.decode("utf-8")

    def push(self, data, final=False):
        """incrementalText.Push: text decodable after these bytes."""
        b = bytes(data)
        return self._call(A.lib().sr_text_decoder_push, (self.h, b, len(b), int(final)), len(b))

    def push_token(self, token_id, piece, final=False):
        """PushToken for one sampled token and its piece."""
        b = bytes(piece)
        return self._call(A.lib().sr_text_decoder_push_token, (self.h, int(token_id), b, len(b), int(final)), len(b))


def _bench(tokens=200_000, seed=0):
    """Host throughput of PushToken on a seeded stream of ByteLevel-like pieces
    (1-4 bytes, some multi-byte characters split across tokens)."""
    import time
    rng = np.random.default_rng(seed)
    text = "".join(rng.choice(list("abcde fghij.,'é€🌀日本")) for _ in range(tokens * 2)).encode()
    cuts = np.sort(rng.choice(len(text), size=tokens - 1, replace=False))
    pieces = [text[a:b] for a, b in zip(np.r_[0, cuts], np.r_[cuts, len(text)])]
    for name, kw in (("plain", {}), ("hf", dict(hf=True)), ("hf+cleanup", dict(hf=True, cleanup=True))):
        d = TextDecoder(**kw)
        t0 = time.perf_counter()
        out = [d.push_token(i, p, i == len(pieces) - 1) for i, p in enumerate(pieces)]
        dt = time.perf_counter() - t0
        assert "".join(out) == TextDecoder(**kw).push(text, True)
        print(f"{name:11s} {len(pieces) / dt:12,.0f} tokens/s  ({dt * 1e6 / len(pieces):.2f} us per token, "
              f"{len(text) / dt / 1e6:.1f} MB/s, Python call included)")


if __name__ == "__main__":
    import sys
    if "--bench" in sys.argv:
        _bench()
