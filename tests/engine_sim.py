"""Engine actor loop over the CPU oracle (test infrastructure).

A pure-Python restatement of Engine.run's integer decisions
(cmd/monolith/monolith.go:8211-8476): admission with whole-page reservations
(M:8348-8361), scheduleTokens (M:8180-8210), lazily acquired LIFO pages
(pagePool.acquire M:5854-5866, KVCache.Close M:6044-6062), one prefillSelected
per tick, sampleWithBlocked for sessions whose prompt is consumed, and
finishing on EOS or max_tokens.  Small cases only: every step runs on the
oracle.
"""

import numpy as np


def simulate(model, requests, limit, max_batch, budget, chunk, mixed_chunk, eos_id=-1, blocked=-1, threads=4):
    """requests: list of dicts(ids, max_tokens, temperature, top_k, top_p, penalty, seed).
    Returns ({request index: (output ids, reason)}, trace of per-tick (counts, page tables))."""
    from oracle import oracle as O
    pt = model.cfg.page_tokens
    pool = np.zeros(limit * model.page_elements, dtype=np.float32)
    free, allocated, reserved = [], 0, 0
    queue = list(enumerate(requests))
    sessions, rotation, finished, trace = [], 0, {}, []

    def acquire():
        nonlocal allocated
        if free:
            return free.pop()
        allocated += 1
        return allocated - 1

    def close(s):
        nonlocal reserved
        free.extend(s["pages"])
        reserved -= s["reserved"]

    while queue or sessions:
        while len(sessions) < max_batch and queue:
            rid, r = queue.pop(0)
            pages = (len(r["ids"]) + r["max_tokens"] + pt - 1) // pt
            if reserved + pages > limit:
                finished[rid] = ([], "busy")
                continue
            reserved += pages
            sessions.append(dict(rid=rid, req=r, pages=[], reserved=pages, pos=0, cursor=0, output=[],
                                 history=list(r["ids"]), rng=r.get("seed", 1)))
        if not sessions:
            break
        n = len(sessions)
        rem = [len(s["req"]["ids"]) - s["cursor"] for s in sessions]
        counts, total = O.schedule_tokens(rem, budget, chunk, mixed_chunk, rotation % n)
        rotation = (rotation + 1) % n
        chunks, want = [], []
        for i, s in enumerate(sessions):
            ids = s["req"]["ids"]
            want.append(s["cursor"] + counts[i] >= len(ids))
            if s["cursor"] < len(ids):
                chunks.append(list(ids[s["cursor"]:s["cursor"] + counts[i]]))
            else:
                chunks.append([s["output"][-1]])
            needed = (s["pos"] + len(chunks[-1]) + pt - 1) // pt
            while len(s["pages"]) < needed:
                s["pages"].append(acquire())
        trace.append((list(counts), [list(s["pages"]) for s in sessions]))
        logits = model.step(pool, [s["pos"] for s in sessions], chunks, [s["pages"] for s in sessions], want,
                            threads=threads)
        alive = []
        for i, s in enumerate(sessions):
            s["pos"] += len(chunks[i])
            ids = s["req"]["ids"]
            if s["cursor"] < len(ids):
                s["cursor"] += counts[i]
            if s["cursor"] < len(ids):
                alive.append(s)
                continue
            r = s["req"]
            tok, s["rng"] = O.sample(logits[i], s["history"], r.get("temperature", 0.0), r.get("top_k", 0),
                                     r.get("top_p", 1.0), r.get("penalty", 1.0), s["rng"], blocked)
            s["output"].append(tok)
            s["history"].append(tok)
            reason = None
            if eos_id >= 0 and tok == eos_id:
                reason = "eos"
            elif len(s["output"]) == r["max_tokens"]:
                reason = "length"
            if reason:
                close(s)
                finished[s["rid"]] = (list(s["output"]), reason)
            else:
                alive.append(s)
        sessions = alive
    return finished, trace
