#!/usr/bin/env python
"""Benchmark of the engine step: BASELINE config 4, Mistral-7B-shaped Q8.

Workload (one rank = one GPU = one engine): 256 concurrent requests with prompt
lengths log-normal (median 1024, sigma 1.0, capped at 8192), outputs uniform in
64..512, 16-token KV pages, reference default sampling (T 0.8, top-k 40,
top-p 0.95, repeat penalty 1.1) on the SplitMix64 streams.  Weights are a
seeded random init (N(0, 0.02), quantised to Q8 with the reference's block
quantizer) generated on the device.  A "step" is one engine tick in steady
decode: every session appends one token (prefillSelected over 256 decode rows
+ sampleWithBlocked), so output tokens per step = 256.  The KV pages already
hold each session's prompt and the decode tokens before its starting offset
(synthetic values: a prefilled cache); offsets are uniform in the session's
output budget so contexts are ragged, as in a running server.

With --split, a one-GPU fast step of at least 128 rows runs as two halves on two SM
partitions (green contexts), so one half's attention overlaps the other
half's projections (`--split`; `config.step_halves` = 2).
`value`   = output tokens / s over all ranks from the device span of each step
            (first to last kernel, CUDA events on the library's stream).
`e2e`     = the same metric through the C ABI call sr_step_sample with host
            buffers: the step's batch metadata and sampling history are copied
            from pinned host memory and the sampled ids are read back every step;
            timed with events on the same stream around the whole K steps
            (host gaps included).
Multi-GPU (--gpus N under torchrun): the N ranks serve the same 256-request
engine tensor-parallel -- each holds 1/N of the heads, FFN columns and KV pool
and the step all-reduces after o_proj and down_proj over NCCL -- so total
work is fixed (strong scaling).  --parallel replicas runs N independent
engines instead (weak scaling).
`ttft_p50_ms`, `stream_output_tok_s` (and `serving`) come from a serving run
            after the decode measurement: the same 256 requests (prompt ids
            uniform over the vocabulary) are submitted at once to the C++
            restatement of the reference engine (admission, scheduleTokens,
            steps, sampling) on an empty KV pool, with prefill chunks of 1024
            tokens (also while sessions decode: --stream-mixed-chunk, whose
            reference default is 1) and a 1024-row token budget, until the last
            request completes.  TTFT is submit -> first sampled token, host
            clock after the step's synchronising sample call (M:8441-8447);
            stream tok/s = generated tokens / wall time from submission to the
            last completion.
`--impl reference` times the CPU oracle (the C restatement of the reference's
Go step, all host threads): W untimed and K timed steps, each a decode step of
8 of the 256 sessions (a bounded sample of the same workload).
--config qwen7b measures the Qwen2.5-7B long-context configuration instead:
16 sessions with 31,744-token prompts (synthetic prefilled KV pages) decoding
up to 1,024 tokens each, q4-mixed weights, split-K attention over contexts of
31,744..32,768 positions; tensor-parallel 8 ways on 8 GPUs (each KV head on a
pair of ranks that split its 7 query heads 4/3).
"""

import argparse
import ctypes as C
import json
import math
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIG = dict(name="mistral7b-q8-256req", vocab=32768, dim=4096, hidden=14336, layers=32, heads=32, kv_heads=8,
              context=32768, rope_theta=1e6, norm_eps=1e-5, tied=False, qkv_bias=False, fmt="q8", page_tokens=16,
              sessions=256, prompt_median=1024, prompt_sigma=1.0, prompt_max=8192, out_lo=64, out_hi=512,
              sampling=(0.8, 40, 0.95, 1.1), seed=20261201,
              metric="output tok/s, Mistral-7B-shape Q8, 256 ragged reqs; p50 TTFT/ITL; HBM GB/s")
# The Qwen2.5-7B long-context configuration: 16 sessions whose 31,744-token
# prompts leave room for 1,024 decode tokens inside the reference's 32,768
# context (prompt + max_tokens <= Context); decoding through split-K attention.
QWEN7B = dict(name="qwen2.5-7b-q4mixed-16x31744", vocab=152064, dim=3584, hidden=18944, layers=28, heads=28,
              kv_heads=4, context=32768, rope_theta=1e6, norm_eps=1e-6, tied=False, qkv_bias=True, fmt="q4-mixed",
              page_tokens=16, sessions=16, prompt_fixed=31744, out_lo=1024, out_hi=1024,
              sampling=(0.8, 40, 0.95, 1.1), seed=20261202,
              metric="output tok/s, Qwen2.5-7B-shape q4-mixed, 16 x 31,744-token prompts decoding 1,024; HBM GB/s")
CONFIGS = {"mistral7b": CONFIG, "qwen7b": QWEN7B}
METRIC = CONFIG["metric"]


def workload(cfg, rank, warmup_steps):
    rng = np.random.default_rng(cfg["seed"] + 7919 * rank)
    S = cfg["sessions"]
    if "prompt_fixed" in cfg:
        prompts = np.full(S, cfg["prompt_fixed"], dtype=np.int64)
    else:
        prompts = np.clip(np.round(np.exp(np.log(cfg["prompt_median"]) + cfg["prompt_sigma"] *
                                          rng.standard_normal(S))), 1, cfg["prompt_max"]).astype(np.int64)
    outs = rng.integers(cfg["out_lo"], cfg["out_hi"] + 1, size=S)
    offsets = np.array([rng.integers(0, max(1, o - warmup_steps)) for o in outs], dtype=np.int64)
    return prompts, outs, offsets, rng


def clocks_start(path, device):
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    try:
        return subprocess.Popen(["nvidia-smi", "-i", str(device), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                 "-lms", "200"], stdout=open(path, "w"), stderr=subprocess.DEVNULL)
    except Exception:
        return None


def clocks_stop(proc, path):
    if proc is None:
        return None
    proc.terminate()
    try:
        proc.wait(timeout=5)
    except Exception:
        proc.kill()
    sm, mx, reasons = [], 0.0, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in open(path):
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9:
            continue
        try:
            sm.append(float(f[1]))
            mx = max(mx, float(f[2]))
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def traffic_per_position():
    """DRAM bytes per (position, layer) of the attention kernel from a committed
    ncu summary, if one exists (profiles/attention_traffic.json)."""
    p = os.path.join(ROOT, "profiles", "attention_traffic.json")
    try:
        return json.load(open(p))
    except Exception:
        return None


def advance_sessions(pos, hist, hoff, ids, prompts, outs):
    """Host bookkeeping after one decode step: each session's sampled id joins
    its history and its position advances.  A session that has used its whole
    output budget (prompt + outs positions) restarts decoding right after its
    prompt, as a fresh request in its slot would, so the step keeps its shape
    and its pages for any number of steps.  Returns (pos, hist, hoff)."""
    hist = np.insert(hist, hoff[1:], ids)  # append each session's new id
    hoff = hoff + np.arange(len(hoff), dtype=np.int32)
    pos = pos + 1
    done = np.nonzero(pos >= prompts + outs)[0]
    if done.size:
        keep = np.ones(hist.size, dtype=bool)
        for i in done:
            keep[hoff[i] + int(prompts[i]):hoff[i + 1]] = False
        lens = np.diff(hoff)
        lens[done] = prompts[done]
        hist = hist[keep]
        hoff = np.zeros_like(hoff)
        hoff[1:] = np.cumsum(lens)
        pos = pos.copy()
        pos[done] = prompts[done]
    return pos.astype(np.int32), hist, hoff.astype(np.int32)


class DecodeState:
    """The workload's sessions in steady decode over one device model and page pool."""

    def __init__(self, cfg, model, warmup, workload_rank=0, steps=0):
        """steps: the decode steps that follow the warm-up; the sessions' starting
        offsets leave room for all of them where the output budget allows."""
        from sr_go_tranformer_b200 import _abi as A
        from sr_go_tranformer_b200 import step as S
        self.A, self.S, self.cfg = A, S, cfg
        prompts, outs, offsets, rng = workload(cfg, workload_rank, warmup + steps)
        self.prompts, self.outs = prompts, outs
        n = cfg["sessions"]
        pt = cfg["page_tokens"]
        self.model = model
        reserve = int(np.sum((prompts + outs + pt - 1) // pt))
        self.pool = S.PagePool(self.model, reserve)
        self.pool.fill_synthetic(cfg["seed"] + 1, 0.5)
        self.pos = (prompts + offsets).astype(np.int32)
        # LIFO page acquisition in session order, as the engine admits them.
        self.pages = [[] for _ in range(n)]
        for i in range(n):
            need = (int(self.pos[i]) + 1 + pt - 1) // pt
            while len(self.pages[i]) < need:
                self.pages[i].append(self.pool.acquire())
        self.page_arr = [np.asarray(p, dtype=np.int32) for p in self.pages]
        V = cfg["vocab"]
        hist = [rng.integers(0, V, size=int(self.pos[i])).astype(np.int32) for i in range(n)]
        self.hist = np.concatenate(hist)  # every session's history, back to back
        self.hoff = np.zeros(n + 1, dtype=np.int32)
        self.hoff[1:] = np.cumsum([len(h) for h in hist])
        self.last = rng.integers(0, V, size=n).astype(np.int32)
        self.rng_state = np.array([cfg["seed"] + i for i in range(n)], dtype=np.uint64)
        t, k, p, pen = cfg["sampling"]
        self.settings = (A.Sampling * n)(*[A.Sampling(t, k, 0, p, pen) for _ in range(n)])
        self.toff = np.arange(n + 1, dtype=np.int32)
        self.ids = np.zeros(n, dtype=np.int32)
        self.n = n
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.ctx_trace = []

    def step(self):
        A, n, pt = self.A, self.n, self.cfg["page_tokens"]
        for i in range(n):  # ensurePages for the new row (lazy LIFO acquire)
            if (int(self.pos[i]) + 1 + pt - 1) // pt > len(self.pages[i]):
                self.pages[i].append(self.pool.acquire())
                self.page_arr[i] = np.asarray(self.pages[i], dtype=np.int32)
        poff = np.zeros(n + 1, dtype=np.int32)
        poff[1:] = np.cumsum([len(p) for p in self.pages])
        pids = np.concatenate(self.page_arr)
        hoff, hist = self.hoff, self.hist
        b = A.Batch(n, self.pos.ctypes.data, self.toff.ctypes.data, self.last.ctypes.data, poff.ctypes.data,
                    pids.ctypes.data, None)
        self.ctx_trace.append(int(np.sum(self.pos.astype(np.int64) + 1)))
        A.check(A.lib().sr_step_sample(self.model.h, self.pool.h, C.byref(b), C.cast(self.settings, C.c_void_p),
                                       hoff.ctypes.data, hist.ctypes.data, self.rng_state.ctypes.data, -1,
                                       self.ids.ctypes.data))
        # bytes crossing the host boundary this step (sr_upload_batch + sampler staging)
        self.h2d_bytes += 4 * (1864 + pids.size) + n * 32 + 4 * (n + 1) + 4 * hist.size + 8 * n
        self.d2h_bytes += 8 * n + 4 * n + 4 * n
        self.pos, self.hist, self.hoff = advance_sessions(self.pos, hist, hoff, self.ids, self.prompts, self.outs)
        self.last[:] = self.ids

    def profile(self, reset=False):
        A = self.A
        ms = (C.c_double * len(A.PROF_CLASSES))()
        la = (C.c_int64 * len(A.PROF_CLASSES))()
        span, steps, total = C.c_double(), C.c_int64(), C.c_int64()
        A.check(A.lib().sr_profile_read(self.model.h, ms, la, C.byref(span), C.byref(steps), C.byref(total),
                                        1 if reset else 0))
        return list(ms), list(la), span.value, steps.value, total.value

    def set_profile(self, mask):
        self.A.check(self.A.lib().sr_profile_set(self.model.h, mask))

    def stream(self):
        s = C.c_void_p()
        self.A.check(self.A.lib().sr_model_stream(self.model.h, C.byref(s)))
        return s.value


def make_model(cfg, device, mode, tp=(0, 1, None)):
    from sr_go_tranformer_b200 import step as S
    d = S.make_desc(cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                    cfg["context"], cfg["rope_theta"], cfg["norm_eps"], cfg["tied"], cfg["qkv_bias"], cfg["fmt"],
                    cfg["page_tokens"])
    model = S.Model(d, device, tp_rank=tp[0], tp_size=tp[1], nccl_id=tp[2])
    model.init_synthetic(cfg["seed"], 0.02)
    model.set_mode(mode)
    return model


def serve_phase(cfg, model, workload_rank=0, mixed_chunk=1024, max_ticks=20000):
    """Serve the workload's 256 requests from an empty pool through the C++
    engine (sr_engine_*) until the last one completes: TTFT (submit -> first
    sampled token) and ITL medians from the engine's own clock, and the
    stream-level output tok/s = all generated tokens / wall time from
    submission to the last completion."""
    from sr_go_tranformer_b200.engine import Engine
    prompts, outs, _, _ = workload(cfg, workload_rank, 0)
    n, pt, V = cfg["sessions"], cfg["page_tokens"], cfg["vocab"]
    pages = int(np.sum((prompts + outs + pt - 1) // pt))
    eng = Engine(model, max_batch=n, token_budget=1024, prefill_chunk=1024, mixed_prefill_chunk=mixed_chunk,
                 cache_bytes=pages * model.page_elements * 4)
    ids_rng = np.random.default_rng(cfg["seed"] + 17)
    t, k, p, pen = cfg["sampling"]
    for i in range(n):
        eng.submit(ids_rng.integers(0, V, size=int(prompts[i])), int(outs[i]), t, k, p, pen, seed=cfg["seed"] + i)
    t0 = time.time()
    ticks = rows = 0
    first_wall = None
    done = 0
    while ticks < max_ticks:
        rows += eng.tick()
        ticks += 1
        while eng.poll() is not None:
            done += 1
        if first_wall is None and eng.latency()["first_tokens"] >= n:
            first_wall = time.time() - t0
        if done >= n:
            break
    wall = time.time() - t0
    lat = eng.latency()
    st = eng.stats()
    eng.close()
    return {"ttft_p50_ms": lat["ttft_p50_ms"], "itl_p50_ms": lat["itl_p50_ms"], "first_tokens": lat["first_tokens"],
            "all_first_tokens_s": first_wall, "completed": done, "ticks": ticks, "wall_s": wall,
            "prompt_tokens": int(np.sum(prompts)), "generated_tokens": int(st["generated_tokens"]),
            "stream_output_tok_s": st["generated_tokens"] / wall, "input_tok_s": st["input_tokens"] / wall,
            "rows": rows, "settings": f"prefill chunk 1024, mixed prefill chunk {mixed_chunk} (the reference default is"
                                      f" 1), token budget 1024, max batch 256, run to the last completion"}


def weight_bytes(cfg):
    """Matrix bytes read once per step (codes + fp32 scales per 64-column
    block; Q4 codes two per byte, the head Q8 under q4-mixed), embedding excluded."""
    d, kd, h, V, L = cfg["dim"], cfg["dim"] // cfg["heads"] * cfg["kv_heads"], cfg["hidden"], cfg["vocab"], cfg["layers"]
    q4 = cfg["fmt"] in ("q4", "q4-mixed")

    def mat(r, c, q4m):
        return r * ((c + 1) // 2 if q4m else c) + r * ((c + 63) // 64) * 4

    mats = [(d, d), (kd, d), (kd, d), (d, d), (h, d), (h, d), (d, h)]
    per_layer = sum(mat(r, c, q4) for r, c in mats) + 2 * d * 4 + (d + 2 * kd) * 4 * cfg.get("qkv_bias", False)
    head = mat(V, d, cfg["fmt"] == "q4")
    return L * per_layer + head + d * 4


def cpu_baseline(cfg, sample_sessions, threads, steps=1, warmup=0):
    """Time the CPU oracle on `sample_sessions` sessions of the same workload:
    `warmup` untimed then `steps` timed decode steps (each session appends one
    token per step)."""
    from oracle import oracle as O
    O.build()
    pt = cfg["page_tokens"]
    c = O.make_config(cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                      cfg["context"], cfg["rope_theta"], cfg["norm_eps"], cfg["tied"], cfg["qkv_bias"], cfg["fmt"], pt)
    m = O.Model(c)
    t0 = time.time()
    m.init_synthetic(cfg["seed"], 0.02, threads=threads)
    init_s = time.time() - t0
    prompts, outs, offsets, rng = workload(cfg, 0, 3)
    idx = list(range(sample_sessions))
    pos = [int(prompts[i] + offsets[i]) for i in idx]
    total = warmup + steps
    tables, nxt = [], 0
    for p in pos:
        k = (p + total + pt - 1) // pt  # pages for every step's position
        tables.append(list(range(nxt, nxt + k)))
        nxt += k
    pool = np.zeros(nxt * m.page_elements, dtype=np.float32)
    toks = [[int(t)] for t in rng.integers(0, cfg["vocab"], size=len(idx))]
    times = []
    for s in range(total):
        t0 = time.time()
        logits = m.step(pool, [p + s for p in pos], toks, tables, threads=threads)
        dt = time.time() - t0
        if s >= warmup:
            times.append(dt)
        toks = [[int(np.argmax(x))] for x in logits]
    t = float(np.sum(times))
    return {"value": len(idx) * steps / t, "unit": "output tok/s", "cores": threads, "kind": "port",
            "sample": f"{len(idx)} of the workload's {cfg['sessions']} sessions (contexts {min(pos)}..{max(pos)}), {warmup} untimed + "
                      f"{steps} timed decode steps, C oracle restating the Go step, {threads} threads; model init "
                      f"{init_s:.1f}s untimed",
            "step_s": t / steps, "steps": steps}


def bench_config(cfg, args, world, tp):
    """The `config` object of the JSON line (both arms report the same one)."""
    return {"workload": cfg["name"], "sessions": cfg["sessions"], "layers": cfg["layers"],
            "page_tokens": cfg["page_tokens"],
            "weights": {"q8": "q8 (64-col blocks, fp32 scales)",
                        "q4-mixed": "q4-mixed (q4 layers, q8 embedding/head; 64-col blocks, fp32 scales)"}[cfg["fmt"]],
            "mode": args.mode, "parallelism": f"tp{world}" if tp else f"replicas{world}",
            "allreduce": (args.allreduce if tp else None),
            "kv_state": "synthetic prefilled pages (prompt + decode offset)",
            "l2": "inputs larger than L2 (KV pool > 100 GB)",
            "sampling": "T0.8 k40 p0.95 penalty1.1, SplitMix64"}


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    W, K = args.warmup, args.steps
    tp = args.gpus > 1 and args.parallel == "tp"
    if args.allreduce == "auto":
        args.allreduce = "peer" if args.gpus == 2 else "nccl"
    from oracle import oracle as O
    O.build()
    # bounded sample: each step is one decode step of 8 of the sessions (about
    # 1.5-2 s of CPU work on 16 cores for config 4), W untimed then K timed
    res = cpu_baseline(cfg, args.ref_sessions, threads, steps=K, warmup=W)
    line = {"impl": "reference", "metric": cfg["metric"], "value": res["value"], "unit": "output tok/s", "n_gpus": args.gpus,
            "steps": res["steps"], "warmup": W, "ms_per_step": res["step_s"] * 1000.0, "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(bench_config(cfg, args, args.gpus, tp), sessions_sampled=args.ref_sessions,
                           sample=f"each step decodes {args.ref_sessions} of the {cfg['sessions']} sessions on the CPU"),
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": "output tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default=os.environ.get("SR_BENCH_MODE", "fast"), choices=["exact", "fast"])
    ap.add_argument("--config", default="mistral7b", choices=sorted(CONFIGS),
                    help="mistral7b: 256 ragged requests, Mistral-7B shape, Q8 (the headline); qwen7b: 16 sessions of "
                         "31,744-token prompts decoding, Qwen2.5-7B shape, q4-mixed")
    ap.add_argument("--sessions", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--cpu-sessions", type=int, default=8)
    ap.add_argument("--ref-sessions", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", default="tp", choices=["tp", "replicas"])
    ap.add_argument("--allreduce", default="auto", choices=["auto", "peer", "peer-ll", "nccl"],
                    help="tensor-parallel all-reduce: the library's NVLink peer-memory kernels (flag barriers, or "
                         "peer-ll: flags inside the data, one kernel), NCCL, or auto (peer at 2 ranks, NCCL above: the "
                         "faster one measured at each size)")
    ap.add_argument("--no-ttft", action="store_true", help="skip the serving run (TTFT, ITL, stream tok/s)")
    ap.add_argument("--split", action="store_true",
                    help="run a one-GPU fast step of >= 128 rows as two halves on two SM partitions, overlapping one "
                         "half's attention with the other's projections")
    ap.add_argument("--stream-mixed-chunk", type=int, default=1024,
                    help="mixed prefill chunk of the serving run (1 = the reference default; slower: with any session "
                         "decoding, every prompt advances one token per tick)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    cfg["sessions"] = args.sessions or cfg["sessions"]
    cfg["layers"] = args.layers or cfg["layers"]
    if args.config != "mistral7b":
        args.no_ttft = True  # the serving run would prefill 16 x 31,744 tokens first
    if args.impl == "reference":
        return run_reference(args, cfg)
    W = max(3, args.warmup)
    K = args.steps
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    torch.cuda.set_device(local)
    dist = None
    tp = world > 1 and args.parallel == "tp"
    tp_args = (0, 1, None)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        if tp:
            from sr_go_tranformer_b200 import step as S
            obj = [S.tp_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            tp_args = (rank, world, obj[0])
    model = make_model(cfg, local, args.mode, tp=tp_args)
    model.set_split(args.split)
    if args.allreduce == "auto":
        args.allreduce = "peer" if world == 2 else "nccl"
    if tp and args.allreduce in ("peer", "peer-ll"):
        handles = [None] * world
        dist.all_gather_object(handles, model.tp_peer_handle())
        model.tp_peer_open(handles)
        if args.allreduce == "peer-ll":
            model.tp_peer_set_protocol("ll")
    st = DecodeState(cfg, model, W, workload_rank=0 if tp else rank, steps=K + 1)  # + the profiled step
    for _ in range(W):
        st.step()
    ext = torch.cuda.ExternalStream(st.stream())
    st.profile(reset=True)
    st.set_profile(1 << 5)  # attention launches timed with events inside the timed region
    st.ctx_trace.clear()
    st.h2d_bytes = st.d2h_bytes = 0
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    tmp = tempfile.NamedTemporaryFile(suffix=".csv", delete=False).name
    clk = clocks_start(tmp, local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(K):
        st.step()
    e1.record(ext)
    torch.cuda.synchronize()
    clocks = clocks_stop(clk, tmp)
    e2e_ms = e0.elapsed_time(e1)
    ctx_trace, h2d, d2h = list(st.ctx_trace), st.h2d_bytes, st.d2h_bytes  # the timed steps only
    ms, launches, span_ms, nsteps, total_launches = st.profile(reset=True)
    st.set_profile(0)
    # Per-class breakdown from a separately profiled step (not timed).
    st.set_profile((1 << 9) - 1)
    st.step()
    cls_ms, cls_launch, _, _, _ = st.profile(reset=True)
    st.set_profile(0)
    # The serving run for TTFT comes after the decode measurement (its prefill
    # steps heat the GPU) and needs the memory of the decode state's KV pool.
    st.pool.close()
    ttft = None if args.no_ttft else serve_phase(cfg, model, workload_rank=0 if tp else rank,
                                                 mixed_chunk=args.stream_mixed_chunk)
    t = torch.tensor([span_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    span_max, e2e_max = float(t[0]), float(t[1])
    tokens = cfg["sessions"] * K * (1 if tp else world)
    value = tokens / (span_max / 1000.0)
    e2e_val = tokens / (e2e_max / 1000.0)
    if rank == 0:
        peaks, peak_kind = measured_peaks()
        kvd = model.kv_dim  # this rank's KV width
        kv_pos_bytes = 2 * kvd * 4  # K + V row of one position, one layer
        attn_launches = launches[5]
        attn_ms = ms[5] / max(1, attn_launches)
        positions = float(np.mean(ctx_trace))  # sum over sessions of (pos+1) per step
        # a launch covers one layer of the whole step, or of one half of a split step
        halves = max(1, round(attn_launches / max(1, cfg["layers"] * K)))
        attn_bytes = (positions * kv_pos_bytes + 2 * cfg["sessions"] * cfg["dim"] * 4) / halves
        achieved = attn_bytes / (attn_ms / 1000.0) / 1e9
        tr = traffic_per_position() if args.config == "mistral7b" else None  # captured on the config-4 shape
        kv_share = kvd / (cfg["dim"] // cfg["heads"] * cfg["kv_heads"])
        traffic = None if tr is None else float(tr["bytes_per_position_layer"] * kv_share * positions +
                                                tr.get("fixed_bytes", 0)) / halves
        wbytes = weight_bytes(cfg) / (world if tp else 1)  # this rank's share (embedding/head replicated: approx)
        step_bytes = wbytes + cfg["layers"] * (positions * kv_pos_bytes + cfg["sessions"] * kv_pos_bytes) + \
            4 * cfg["sessions"] * cfg["vocab"]
        cls_total = sum(cls_ms) or 1.0
        line = {
            "metric": cfg["metric"], "value": value, "unit": "output tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": span_max / K, "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": ("f32; projections bf16 hi+lo x bf16 codes on tensor cores, fp32 accumulate" if args.mode == "fast"
                      else "f32"),
            "data": "synthetic",
            "config": dict(bench_config(cfg, args, world, tp), step_halves=halves),
            "itl_p50_ms": span_max / K, "ttft_p50_ms": ttft["ttft_p50_ms"] if ttft else None,
            "stream_output_tok_s": ttft["stream_output_tok_s"] if ttft else None,
            "hbm_gbs_step": step_bytes / (span_max / K / 1000.0) / 1e9,
            "algorithmic_bytes_per_step": step_bytes,
            "e2e": {"value": e2e_val, "unit": "output tok/s",
                    "h2d_bytes_per_step": h2d // max(1, K), "d2h_bytes_per_step": d2h // max(1, K)},
            "gpu_launches": int(total_launches),
            "roofline": {"kernel": "attention", "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                         "peak_source": peak_kind, "launch_ms": attn_ms, "algorithmic_bytes": attn_bytes},
            "kernels": {n: {"ms_per_step": cls_ms[i], "share": cls_ms[i] / cls_total, "launches": cls_launch[i]}
                        for i, n in enumerate(st.A.PROF_CLASSES)},
            "clocks": clocks,
        }
        if ttft:
            line["serving"] = ttft
        if world == 1 and not args.no_cpu_baseline:
            try:
                cb = cpu_baseline(cfg, args.cpu_sessions, os.cpu_count() or 1)
                line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
            except Exception as e:  # reported, never silently replaced
                line["cpu_baseline"] = {"error": str(e)}
        print(json.dumps(line))
    if dist:
        dist.barrier()
    model.close()  # every rank: the peer all-reduce's last barrier
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
