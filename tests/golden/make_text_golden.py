"""Golden vectors for streaming detokenization, from the reference's tokenizer fixtures.

For every `testdata/hf-*-tokenizer` directory of a reference checkout this
writes, into `text_decode.json` next to itself, the decoder flags the reference
derives (newTextDecoder, cmd/monolith/monolith.go:7662-7668: HF ByteLevel,
`clean_up_tokenization_spaces`, Mistral) and each `decode_cases` entry of the
fixture's reference.json (ids and the string Transformers decoded) together with
the pieces of those ids, built the way hfTokenizer builds them:
  * ByteLevel BPE (M:1850-1872): a vocabulary word maps back to bytes through
    the GPT-2 byte alphabet (hfByteAlphabet, M:1626-1640); a non-special added
    token is its content; special tokens are empty;
  * Mistral (M:2013-2044): "\\u2581" becomes a space, <0xNN> is the byte NN and
    is flagged as byte fallback, special tokens are empty.
Tokenization itself is not restated: only the id -> bytes table is needed.

Usage:  python tests/golden/make_text_golden.py <reference checkout root>
"""

import json
import os
import sys

FIXTURES = ["hf-tokenizer", "hf-gpt2-tokenizer", "hf-llama3-tokenizer", "hf-qwen-tokenizer", "hf-mistral-tokenizer"]


def byte_alphabet_reverse():
    reverse, extra = {}, 256
    for i in range(256):
        r = i
        if not (33 <= i <= 126 or 161 <= i <= 172 or i >= 174):
            r = extra
            extra += 1
        reverse[chr(r)] = i
    return reverse


def pieces_for(tok, mistral):
    vocab = tok["model"]["vocab"]
    added = {a["id"]: a for a in tok.get("added_tokens", [])}
    pieces, fallback = {}, {}
    rev = byte_alphabet_reverse()
    for word, i in vocab.items():
        if i in added:
            a = added[i]
            pieces[i] = b"" if a["special"] else a["content"].encode()
            continue
        if mistral:
            if len(word) == 6 and word.startswith("<0x") and word.endswith(">"):
                pieces[i] = bytes([int(word[3:5], 16)])
                fallback[i] = True
            else:
                pieces[i] = word.replace("▁", " ").encode()
        else:
            pieces[i] = bytes(rev[ch] for ch in word)
    for i, a in added.items():  # added tokens outside the model vocabulary
        if i not in pieces:
            pieces[i] = b"" if a["special"] else a["content"].encode()
    return pieces, fallback


def convert(root, name):
    d = os.path.join(root, "testdata", name)
    tok = json.load(open(os.path.join(d, "tokenizer.json"), encoding="utf-8"))
    cfg = json.load(open(os.path.join(d, "tokenizer_config.json"), encoding="utf-8"))
    ref = json.load(open(os.path.join(d, "reference.json"), encoding="utf-8"))
    mistral = name == "hf-mistral-tokenizer"
    pieces, fallback = pieces_for(tok, mistral)
    cases = []
    for c in ref["decode_cases"]:
        ids = c["ids"]
        cases.append({"ids": ids, "decoded": c["decoded"], "pieces": [pieces.get(i, b"").hex() for i in ids],
                      "fallback": [bool(fallback.get(i, False)) for i in ids]})
    return {"name": name, "hf": True, "cleanup": bool(cfg.get("clean_up_tokenization_spaces", False)),
            "mistral": mistral, "cases": cases}


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SR_REFERENCE_ROOT", "")
    if not root:
        raise SystemExit("usage: make_text_golden.py <reference checkout root>")
    out = [convert(root, f) for f in FIXTURES]
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "text_decode.json")
    with open(path, "w", encoding="utf-8") as f:
        json.dump(out, f, ensure_ascii=False, indent=1)
    print("wrote", path, sum(len(t["cases"]) for t in out), "cases")


if __name__ == "__main__":
    main()
