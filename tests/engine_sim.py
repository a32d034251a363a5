"""Engine actor loop over the CPU oracle (test infrastructure).

A pure-Python restatement of Engine.run's integer decisions
(cmd/monolith/monolith.go:8211-8476): admission with whole-page reservations
(M:8348-8361), scheduleTokens (M:8180-8210), lazily acquired LIFO pages
(pagePool.acquire M:5854-5866, KVCache.Close M:6044-6062), one prefillSelected
per tick, sampleWithBlocked for sessions whose prompt is consumed, and
finishing on EOS or max_tokens.  With prefix_limit > 0 it also keeps the
engine's one-entry prefix snapshot (prefixSnapshot, M:5868-5952): restore at
admission (M:8356), capture when a session finishes (M:8285-8288), snapshot
page i stored as pool page limit + i.  Small cases only: every step runs on
the oracle.
"""

import numpy as np


def simulate(model, requests, limit, max_batch, budget, chunk, mixed_chunk, eos_id=-1, blocked=-1, threads=4,
             prefix_limit=0, prefix_tail=False, stats=None):
    """requests: list of dicts(ids, max_tokens, temperature, top_k, top_p, penalty, seed).
    Returns ({request index: (output ids, reason)}, trace of per-tick (counts, page tables at the
    step, page tables of the sessions still active after the tick)).
    stats, when a dict, receives prefix_hits / prefix_tokens / prefix_pages."""
    from oracle import oracle as O
    pt = model.cfg.page_tokens
    kvd = model.cfg.kv_heads * (model.cfg.dim // model.cfg.heads)
    pe = model.page_elements
    pool = np.zeros((limit + prefix_limit) * pe, dtype=np.float32)
    free, allocated, reserved = [], 0, 0
    queue = list(enumerate(requests))
    sessions, rotation, finished, trace = [], 0, {}, []
    snap = dict(valid=False, ids=[], pages=0, borrowers=0)
    hits = tokens = 0

    def copy_rows(dst, src, rows):
        d, s_ = dst * pe, src * pe
        for off in range(0, pe, pt * kvd):
            pool[d + off:d + off + rows * kvd] = pool[s_ + off:s_ + off + rows * kvd]

    def restore(s):
        ids = s["req"]["ids"]
        if not snap["valid"] or len(ids) < 2:
            return
        n = min(len(snap["ids"]), len(ids) - 1)
        matched = 0
        while matched < n and snap["ids"][matched] == ids[matched]:
            matched += 1
        full = matched // pt
        if full > 0:
            s["pages"] = [limit + i for i in range(full)]
            s["shared"] = full
            snap["borrowers"] += 1
        s["pos"] = full * pt
        if prefix_tail and matched % pt:
            s["pages"].append(acquire())
            copy_rows(s["pages"][full], limit + full, matched % pt)
            s["pos"] = matched

    def capture(s):
        sole = s["shared"] > 0 and snap["borrowers"] == 1 and snap["valid"]
        if snap["borrowers"] != 0 and not sole:
            return
        positions = s["pos"]
        if not prefix_tail:
            positions -= positions % pt
        n = min(prefix_limit, (positions + pt - 1) // pt)
        positions = min(positions, n * pt)
        if n == 0:
            return
        snap["pages"] = max(snap["pages"], n)
        for i in range(n):
            if limit + i != s["pages"][i]:
                copy_rows(limit + i, s["pages"][i], min(pt, positions - i * pt))
        snap["ids"] = list(s["history"][:positions])
        snap["valid"] = True

    def acquire():
        nonlocal allocated
        if free:
            return free.pop()
        allocated += 1
        return allocated - 1

    def close(s):
        nonlocal reserved
        free.extend(s["pages"][s["shared"]:])
        reserved -= s["reserved"]
        if s["shared"]:
            snap["borrowers"] -= 1
            if snap["borrowers"] == 0 and not snap["valid"]:
                snap["pages"] = 0

    while queue or sessions:
        while len(sessions) < max_batch and queue:
            rid, r = queue.pop(0)
            pages = (len(r["ids"]) + r["max_tokens"] + pt - 1) // pt
            if reserved + pages > limit:
                finished[rid] = ([], "busy")
                continue
            reserved += pages
            s = dict(rid=rid, req=r, pages=[], reserved=pages, pos=0, cursor=0, output=[], shared=0,
                     history=list(r["ids"]), rng=r.get("seed", 1))
            if prefix_limit:
                restore(s)
                if s["pos"] > 0:
                    hits += 1
                    tokens += s["pos"]
                s["cursor"] = s["pos"]
            sessions.append(s)
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
                if prefix_limit:
                    capture(s)
                close(s)
                finished[s["rid"]] = (list(s["output"]), reason)
            else:
                alive.append(s)
        trace[-1] = trace[-1] + ([list(s["pages"]) for s in alive],)  # page tables after the tick
        sessions = alive
    if stats is not None:
        stats.update(prefix_hits=hits, prefix_tokens=tokens, prefix_pages=snap["pages"])
    return finished, trace
