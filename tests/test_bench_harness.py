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
