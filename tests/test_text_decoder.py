"""Streaming detokenization (sr_text_decoder_*, host only) on the CPU.

* The plain decoder against the reference's own streaming cases
  (streaming_test.go:23-66): every two-way split and byte-at-a-time feeding
  must equal strings.ToValidUTF8 of the whole string (one replacement per run
  of invalid bytes), emit only valid UTF-8, and a repeated finalisation emits
  nothing.  The expected strings come from Python's UTF-8 decoder with each
  run of invalid bytes collapsed to one U+FFFD.
* The HF / Mistral decoders against the decode cases of the reference's five
  tokenizer fixtures (tests/golden/text_decode.json, made by
  tests/golden/make_text_golden.py): whole decode, every two-way split and
  byte-at-a-time for ByteLevel tokenizers (hf_llama3_tokenizer_test.go:131-158),
  and token-at-a-time PushToken (hf_tokenizer_test.go:125-131).
"""

import codecs
import json
import os

import pytest

from conftest import GOLDEN_DIR

CASES = [
    b"", "cat 猫 🌀 日本語".encode(),
    bytes([ord("a"), 0xFF, 0xFE, ord("b")]),
    bytes([0xE7, 0x8C]),
    bytes([0xFF, 0xE7, 0x8C, 0xAB, 0xFE]),
    bytes([0xED, 0xA0, 0x80, 0xC0, 0xAF, ord("x"), 0x80, 0x81]),
    bytes([0xE7, 0xFF, 0x8C, 0xAB, ord("x"), 0xF0, 0x9F]),
    bytes(range(256)),
]


def _collapse_runs(err):
    # One replacement per run of invalid bytes: a run continues while the
    # decoder reports errors back to back.
    first = not hasattr(_collapse_runs, "end") or _collapse_runs.end != err.start or _collapse_runs.obj is not err.object
    _collapse_runs.end, _collapse_runs.obj = err.end, err.object
    return ("�" if first else "", err.end)


codecs.register_error("sr_collapse_runs", _collapse_runs)


def to_valid_utf8(raw):
    """strings.ToValidUTF8(string(raw), "\\ufffd")."""
    _collapse_runs.end = -1
    _collapse_runs.obj = None
    return bytes(raw).decode("utf-8", "sr_collapse_runs")


def _td():
    from sr_go_tranformer_b200.text import TextDecoder
    return TextDecoder


def test_expected_strings_follow_go_semantics():
    assert to_valid_utf8(bytes([ord("a"), 0xFF, 0xFE, ord("b")])) == "a�b"
    assert to_valid_utf8(bytes([0xE7, 0x8C])) == "�"
    assert to_valid_utf8("�".encode() + b"\xff") == "��"  # a real U+FFFD is not a run


@pytest.mark.parametrize("case", range(len(CASES)))
def test_plain_decoder_streams_like_whole_decode(srlib, case):
    TD = _td()
    raw = CASES[case]
    want = to_valid_utf8(raw)
    for split in range(len(raw) + 1):
        d = TD()
        first = d.push(raw[:split], False)
        last = d.push(raw[split:], True)
        assert first + last == want, (case, split)
        assert d.push(b"", True) == ""
    d = TD()
    got = "".join(d.push(bytes([b]), False) for b in raw) + d.push(b"", True)
    assert got == want


GOLD = json.load(open(os.path.join(GOLDEN_DIR, "text_decode.json"), encoding="utf-8"))


def _decoder(t, cases=None):
    TD = _td()
    fallback = None
    if t["mistral"]:
        ids = [i for c in (cases or t["cases"]) for i in c["ids"]]
        fallback = [0] * (max(ids) + 1)
        for c in (cases or t["cases"]):
            for i, f in zip(c["ids"], c["fallback"]):
                fallback[i] = int(f)
    return TD(hf=t["hf"], cleanup=t["cleanup"], mistral=t["mistral"], fallback=fallback)


@pytest.mark.parametrize("t", GOLD, ids=lambda t: t["name"])
def test_tokenizer_decode_cases_token_at_a_time(srlib, t):
    """PushToken per id, final on the last (hf_tokenizer_test.go:125-131)."""
    for c in t["cases"]:
        d = _decoder(t)
        pieces = [bytes.fromhex(p) for p in c["pieces"]]
        got = "".join(d.push_token(i, p, k == len(pieces) - 1) for k, (i, p) in enumerate(zip(c["ids"], pieces)))
        if t["mistral"]:
            got += d.push_token(-1, b"", True)
        assert got == c["decoded"], (t["name"], c["ids"])


@pytest.mark.parametrize("t", [t for t in GOLD if not t["mistral"]], ids=lambda t: t["name"])
def test_tokenizer_decode_cases_any_split(srlib, t):
    """Concatenated pieces through Push: whole, every two-way split, and byte at
    a time (hf_llama3_tokenizer_test.go:131-158)."""
    for c in t["cases"]:
        raw = b"".join(bytes.fromhex(p) for p in c["pieces"])
        for split in range(len(raw) + 1):
            d = _decoder(t)
            got = d.push(raw[:split], False) + d.push(raw[split:], False) + d.push(b"", True)
            assert got == c["decoded"], (t["name"], c["ids"], split)
        d = _decoder(t)
        got = "".join(d.push(bytes([b]), False) for b in raw) + d.push(b"", True)
        assert got == c["decoded"], (t["name"], c["ids"])


def test_cleanup_cascade_holds_partial_patterns(srlib):
    """Transformers' cleanup (M:7672-7701) across token boundaries: a pattern
    split between pieces is still replaced, and nothing is held at the end."""
    TD = _td()
    text = "I don 't know . Do n't you ' re sure , right ? Yes !"
    want = text
    for pat, rep in ((" .", "."), (" ?", "?"), (" !", "!"), (" ,", ","), (" ' ", "'"), (" n't", "n't"),
                     (" 'm", "'m"), (" 's", "'s"), (" 've", "'ve"), (" 're", "'re")):
        want = want.replace(pat, rep)
    raw = text.encode()
    for step in (1, 2, 3, 5):
        d = TD(hf=True, cleanup=True)
        got = "".join(d.push(raw[i:i + step], False) for i in range(0, len(raw), step)) + d.push(b"", True)
        assert got == want, step


def test_mistral_leading_space_and_fallback_runs(srlib):
    TD = _td()
    fb = [0] * 8
    fb[5] = fb[6] = 1  # byte-fallback ids
    d = TD(hf=True, mistral=True, fallback=fb)
    out = d.push_token(1, b" Hello", False)
    assert out == "Hello"  # one leading space stripped, once
    assert d.push_token(2, b" world", False) == " world"
    assert d.push_token(5, b"\xe2", False) == ""  # run pending
    assert d.push_token(6, b"\x82", False) == ""
    assert d.push_token(5, b"\xac", False) == ""
    assert d.push_token(3, b"!", True) == "€!"  # valid run flushed whole
    d = TD(hf=True, mistral=True, fallback=fb)
    assert d.push_token(5, b"\xe2", False) == ""
    assert d.push_token(6, b"\x82", True) == "��"  # invalid run: one per byte


def test_errors(srlib):
    from sr_go_tranformer_b200 import _abi as A
    import ctypes as C
    h = C.c_void_p()
    assert A.lib().sr_text_decoder_create(A.SR_TEXT_CLEANUP, None, 0, C.byref(h)) == A.SR_EINVAL
    assert A.lib().sr_text_decoder_create(64, None, 0, C.byref(h)) == A.SR_EINVAL
    assert A.lib().sr_text_decoder_create(A.SR_TEXT_MISTRAL, None, 10, C.byref(h)) == A.SR_EINVAL


def _random_pieces(rng, data):
    cuts = sorted(rng.choice(len(data) + 1, size=min(len(data), int(rng.integers(0, 8))), replace=False)) if data else []
    out, prev = [], 0
    for c in list(cuts) + [len(data)]:
        out.append(data[prev:c])
        prev = c
    return out


def test_random_streams_split_anywhere(srlib):
    """Property check over seeded random byte streams (ASCII, multi-byte
    sequences, truncated and invalid bytes, cleanup patterns): pieces cut at
    random points decode to the same text as the whole stream, for the plain,
    HF and HF+cleanup decoders; the plain decoder equals ToValidUTF8."""
    import numpy as np
    TD = _td()
    rng = np.random.default_rng(2024)
    alphabet = [b"a", b" ", b".", b"'", b"s", b"n't", b"\xc3\xa9", b"\xe2\x82\xac", b"\xf0\x9f\x8c\x80", b"\xe2\x82",
                b"\xf0\x9f", b"\xff", b"\x80", b"\xc0", b"\xed\xa0\x80", b" 're", b" ,", b" !"]
    for _ in range(300):
        data = b"".join(alphabet[int(i)] for i in rng.integers(0, len(alphabet), size=int(rng.integers(0, 24))))
        pieces = _random_pieces(rng, data)
        for kw in (dict(), dict(hf=True), dict(hf=True, cleanup=True)):
            whole = TD(**kw).push(data, True)
            d = TD(**kw)
            got = "".join(d.push(p, False) for p in pieces) + d.push(b"", True)
            assert got == whole, (kw, data, pieces)
        assert TD().push(data, True) == to_valid_utf8(data), data
        assert TD(hf=True).push(data, True) == data.decode("utf-8", "replace"), data
