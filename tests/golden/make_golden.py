"""Convert the reference's Transformers golden fixtures into compact .npz files.

The reference pins its inference step against tiny random-init Hugging Face
models whose logits and per-layer K/V were produced by Transformers 4.57.1
(`testdata/hf-{llama,llama3,qwen2,mistral}/<variant>/{config.json,
model.safetensors, reference.json}`, checked by
`cmd/monolith/hf_inference_test.go:32-130` at abs tolerance 2e-5).  This script
reads those fixtures from a reference checkout and writes one `<family>-<variant>.npz`
per fixture next to itself, holding:

  config      JSON string of the HF config
  param_<i>   fp32 weights in the reference's hfProfileSpecs order
              (cmd/monolith/monolith.go:407-442), widened from F16/BF16 exactly
              as the reference loader does
  ids         int32[37] prompt ids
  logits      float32[37, vocab]
  cache_k/v   float32[layers, 37, kv_dim]
  weight_sha256  the fixture's pinned weight digest (checked here)

The GPT-2 fixtures (`testdata/hf-gpt2/{legacy-f32,f16,bf16}`) go to
`gpt2/hf-gpt2-<variant>.npz` in loadGPT2's parameter order
(cmd/monolith/monolith.go:5052-5165): the Conv1D weights ([in, out]) are
transposed to [out, in], c_attn is split into q, k, v and its bias likewise, and
the legacy causal-mask tensors are checked (ones on and below the diagonal)
and dropped.  They sit in a subfolder because the device step does not run the
GPT-2 profile yet.

Usage:  python tests/golden/make_golden.py <reference checkout root>
"""

import hashlib
import json
import os
import struct
import sys

import numpy as np

FIXTURES = [
    "hf-llama/f32", "hf-llama/f16", "hf-llama/bf16", "hf-llama/untied-f32",
    "hf-llama3/f32", "hf-llama3/f16", "hf-llama3/bf16",
    "hf-qwen2/f32", "hf-qwen2/f16", "hf-qwen2/untied-bf16",
    "hf-mistral/f32", "hf-mistral/f16", "hf-mistral/bf16",
]
GPT2_FIXTURES = ["hf-gpt2/legacy-f32", "hf-gpt2/f16", "hf-gpt2/bf16"]


def read_safetensors(path):
    raw = open(path, "rb").read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + hlen])
    base = 8 + hlen
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        lo, hi = info["data_offsets"]
        buf = raw[base + lo:base + hi]
        dt = info["dtype"]
        if dt == "F32":
            arr = np.frombuffer(buf, dtype="<f4").astype(np.float32)
        elif dt == "F16":
            arr = np.frombuffer(buf, dtype="<f2").astype(np.float32)
        elif dt == "BF16":
            u16 = np.frombuffer(buf, dtype="<u2").astype(np.uint32)
            arr = (u16 << 16).view(np.float32)
        else:
            raise ValueError(f"unsupported dtype {dt}")
        out[name] = arr.reshape(info["shape"])
    return out


def spec_names(cfg):
    """hfProfileSpecs order (cmd/monolith/monolith.go:407-442)."""
    L = cfg["num_hidden_layers"]
    names = ["model.embed_tokens.weight"]
    for i in range(L):
        p = f"model.layers.{i}."
        names += [p + "input_layernorm.weight", p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                  p + "self_attn.v_proj.weight", p + "self_attn.o_proj.weight",
                  p + "post_attention_layernorm.weight", p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight"]
    names.append("model.norm.weight")
    if cfg["model_type"] == "qwen2":
        for i in range(L):
            p = f"model.layers.{i}.self_attn."
            names += [p + "q_proj.bias", p + "k_proj.bias", p + "v_proj.bias"]
    if not cfg.get("tie_word_embeddings", False):
        names.append("lm_head.weight")
    return names


def gpt2_params(cfg, tensors):
    """loadGPT2's parameter order with [out, in] matrices (M:5052-5165)."""
    t = {k[len("transformer."):] if k.startswith("transformer.") else k: v for k, v in tensors.items()}
    d, L, ctx = cfg["n_embd"], cfg["n_layer"], cfg["n_positions"]
    out = [t["wte.weight"], t["wpe.weight"], t["ln_f.weight"], t["ln_f.bias"]]
    for i in range(L):
        p = f"h.{i}."
        mask = t.get(p + "attn.bias")
        if mask is not None:
            want = np.tril(np.ones((ctx, ctx), dtype=np.float32)).reshape(1, 1, ctx, ctx)
            if not np.array_equal(mask, want):
                raise SystemExit(f"{p}attn.bias: invalid legacy causal mask")
        w = t[p + "attn.c_attn.weight"].T  # [3d, d]
        b = t[p + "attn.c_attn.bias"]
        out += [t[p + "ln_1.weight"], t[p + "ln_1.bias"], w[:d], w[d:2 * d], w[2 * d:], b[:d], b[d:2 * d], b[2 * d:],
                t[p + "attn.c_proj.weight"].T, t[p + "attn.c_proj.bias"], t[p + "ln_2.weight"], t[p + "ln_2.bias"],
                t[p + "mlp.c_fc.weight"].T, t[p + "mlp.c_fc.bias"], t[p + "mlp.c_proj.weight"].T,
                t[p + "mlp.c_proj.bias"]]
    return out


def convert(root, fixture, outdir):
    d = os.path.join(root, "testdata", fixture)
    cfg = json.load(open(os.path.join(d, "config.json")))
    ref = json.load(open(os.path.join(d, "reference.json")))
    wpath = os.path.join(d, "model.safetensors")
    sha = hashlib.sha256(open(wpath, "rb").read()).hexdigest()
    if sha != ref["weight_sha256"]:
        raise SystemExit(f"{fixture}: weight digest mismatch")
    tensors = read_safetensors(wpath)
    arrays = {"config": np.array(json.dumps(cfg)), "weight_sha256": np.array(sha),
              "ids": np.array(ref["ids"], dtype=np.int32),
              "logits": np.array(ref["logits"], dtype=np.float32),
              "cache_k": np.array([c["k"] for c in ref["cache"]], dtype=np.float32),
              "cache_v": np.array([c["v"] for c in ref["cache"]], dtype=np.float32)}
    if cfg["model_type"] == "gpt2":
        for i, a in enumerate(gpt2_params(cfg, tensors)):
            arrays[f"param_{i}"] = np.ascontiguousarray(a.astype(np.float32))
    else:
        for i, name in enumerate(spec_names(cfg)):
            arrays[f"param_{i}"] = np.ascontiguousarray(tensors[name].astype(np.float32))
    name = fixture.replace("/", "-")
    np.savez_compressed(os.path.join(outdir, name + ".npz"), **arrays)
    return name


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SR_REFERENCE_ROOT", "")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout root>")
    outdir = os.path.dirname(os.path.abspath(__file__))
    for f in FIXTURES:
        print("wrote", convert(root, f, outdir))
    os.makedirs(os.path.join(outdir, "gpt2"), exist_ok=True)
    for f in GPT2_FIXTURES:
        print("wrote", convert(root, f, os.path.join(outdir, "gpt2")))


if __name__ == "__main__":
    main()
