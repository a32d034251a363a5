"""The benchmark harness's host bookkeeping (bench.advance_sessions), on CPU:
histories grow by the sampled id, positions advance, and a session that used
its whole output budget restarts after its prompt without new pages, so any
number of timed steps fits the reserved KV pool."""

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def test_advance_appends_and_wraps():
    import bench
    rng = np.random.default_rng(1)
    n = 6
    prompts = rng.integers(1, 20, size=n).astype(np.int64)
    outs = rng.integers(2, 6, size=n).astype(np.int64)
    pos = (prompts + rng.integers(0, 2, size=n)).astype(np.int32)
    hists = [rng.integers(0, 100, size=int(p)).tolist() for p in pos]
    hist = np.concatenate([np.asarray(h, np.int32) for h in hists])
    hoff = np.zeros(n + 1, np.int32)
    hoff[1:] = np.cumsum([len(h) for h in hists])
    for step in range(40):
        ids = rng.integers(0, 100, size=n).astype(np.int32)
        pos, hist, hoff = bench.advance_sessions(pos, hist, hoff, ids, prompts, outs)
        for i in range(n):
            hists[i].append(int(ids[i]))
            if len(hists[i]) >= prompts[i] + outs[i]:
                hists[i] = hists[i][:int(prompts[i])]
            assert hist[hoff[i]:hoff[i + 1]].tolist() == hists[i], (step, i)
            assert pos[i] == len(hists[i])
            assert prompts[i] <= pos[i] < prompts[i] + outs[i]  # within the reserved pages


def test_workloads_stay_inside_the_context():
    """Config 4: log-normal prompts capped at 8192, outputs 64..512.  Config 5
    (--config qwen7b): 16 prompts of 31,744 tokens with 1,024 decode tokens, so
    every position a warm-up, timed or profiled step reaches is below the
    reference's 32,768-position context."""
    import bench
    p, o, off, _ = bench.workload(bench.CONFIG, 0, 3)
    assert len(p) == 256 and p.min() >= 1 and p.max() <= 8192
    assert o.min() >= 64 and o.max() <= 512 and np.all(off < o)
    q = bench.QWEN7B
    p, o, off, _ = bench.workload(q, 0, 3 + 10 + 1)
    assert np.all(p == 31744) and np.all(o == 1024)
    assert np.all(p + off + 3 + 10 + 1 <= q["context"])


def test_weight_bytes_per_step():
    """Matrix bytes read per step (codes + fp32 scales per 64-column block,
    embedding excluded): Mistral-7B Q8 and Qwen2.5-7B q4-mixed (Q4 layers with
    two codes per byte and q/k/v biases, Q8 head)."""
    import bench
    assert bench.weight_bytes(bench.CONFIG) == 7_559_200_768
    q = bench.QWEN7B
    d, h, V, L, kd = 3584, 18944, 152064, 28, 512

    def mat(r, c, q4):
        return r * ((c + 1) // 2 if q4 else c) + r * ((c + 63) // 64) * 4

    layer = sum(mat(r, c, True) for r, c in [(d, d), (kd, d), (kd, d), (d, d), (h, d), (h, d), (d, h)])
    layer += 2 * d * 4 + (d + 2 * kd) * 4  # two norm weights; q/k/v biases (q: d, k and v: kd each)
    want = L * layer + mat(V, d, False) + d * 4
    assert bench.weight_bytes(q) == want


def test_reference_arm_reports_the_steps_it_ran():
    """--impl reference times the CPU oracle for W untimed and K timed steps
    of 8 sessions and prints one JSON line saying so (1-layer copy here)."""
    import json
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--layers", "1",
                          "--steps", "2", "--warmup", "1"], capture_output=True, text=True, timeout=600, check=True)
    line = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 1
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert "1 untimed + 2 timed" in line["cpu_baseline"]["sample"]
