"""Plain-Python statement of the expert-parallel exchange layout (test
infrastructure): what qmoe_ep_dispatch writes on the sending rank and the
(row, slot) numbering qmoe_ep_experts uses for its outputs on the receiving
rank.  The CUDA kernels are checked against it bit for bit, and the CPU
exchange tests use it as their fake device."""
from __future__ import annotations

import numpy as np


def dispatch_plan(idx: np.ndarray, E: int, G: int, placement=None):
    """idx [T][k] global expert ids (-1: failed token); placement[e] (optional)
    = the expert's slot rank * (E/G) + local id, else contiguous shards.  Returns
    (send_tok [rows], send_meta [rows][k], counts [2G], pair_pos [T*k]):
    rows grouped by rank r = e // (E/G), token order inside a rank; the meta
    row holds the expert's local id on r per slot (-1 for slots elsewhere);
    counts = rows per rank then pairs per rank; pair_pos = the pair's place in
    the returned outputs (rank groups in rank order; inside a rank, (row, slot)
    order), -1 for invalid slots."""
    T, k = idx.shape
    eloc = E // G
    if placement is not None:  # expert e lives at slot placement[e] = rank * eloc + local id
        idx = np.where(idx >= 0, np.asarray(placement, dtype=np.int64)[np.maximum(idx, 0)], -1)
    send_tok, send_meta = [], []
    rows, pairs = [0] * G, [0] * G
    local = {}
    for r in range(G):
        for t in range(T):
            js = [j for j in range(k) if idx[t, j] >= 0 and idx[t, j] // eloc == r]
            if not js:
                continue
            meta = [-1] * k
            for j in js:
                meta[j] = int(idx[t, j]) - r * eloc
                local[(t, j)] = (r, pairs[r])
                pairs[r] += 1
            send_tok.append(t)
            send_meta.append(meta)
            rows[r] += 1
    pair_off = np.concatenate([[0], np.cumsum(pairs)[:-1]]).astype(np.int64)
    pair_pos = np.full(T * k, -1, dtype=np.int32)
    for (t, j), (r, q) in local.items():
        pair_pos[t * k + j] = pair_off[r] + q
    meta = np.array(send_meta, dtype=np.int32).reshape(-1, k)
    return np.array(send_tok, dtype=np.int64), meta, np.array(rows + pairs, dtype=np.int32), pair_pos


def pair_rows(meta: np.ndarray):
    """Receiver: (row, local expert) of every valid slot in (row, slot) order."""
    rows, slots = np.nonzero(meta >= 0)
    return rows, meta[rows, slots]
