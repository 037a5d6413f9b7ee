"""Expert-parallel dispatch plan restated in numpy (TEST INFRASTRUCTURE ONLY).

Mirrors the bookkeeping of infer.net_b200/csrc/ep.cuh so that the multi-rank logic can be
checked on CPU ranks: a token is sent once to every rank that owns one of its experts, in
ascending token order per destination; a receiver orders the routes of each of its experts by
(source rank, source row, slot). The claim checked by tests/test_ep_plan_cpu.py: with token
shards contiguous in rank order, this equals the single-GPU stable permutation
(native/DeepInfer.Metal/prefill_moe.mm:12-14 order) restricted to the rank's experts.
"""
import numpy as np


def layout(ids: np.ndarray, E_l: int, G: int):
    """send_idx [T, G] (position of token t among the rows sent to rank d, or -1), counts [G]."""
    T = ids.shape[0]
    dest = ids // E_l
    send_idx = np.full((T, G), -1, np.int64)
    counts = np.zeros(G, np.int64)
    for t in range(T):
        for d in sorted(set(dest[t].tolist())):
            send_idx[t, d] = counts[d]
            counts[d] += 1
    return send_idx, counts


def pack(ids: np.ndarray, tok0: int, E_l: int, G: int):
    """Rows for each destination: (global token, 8 ids) in send order."""
    send_idx, counts = layout(ids, E_l, G)
    rows = [[None] * int(counts[d]) for d in range(G)]
    for t in range(ids.shape[0]):
        for d in range(G):
            if send_idx[t, d] >= 0:
                rows[d][send_idx[t, d]] = (tok0 + t, ids[t].copy())
    return rows, send_idx


def receive_permutation(recv_rows_by_source, rank: int, E_l: int):
    """Concatenate rows in source-rank order; stable-sort the local routes by local expert.
    Returns {local expert: [global route ids]}."""
    rows = [r for src in recv_rows_by_source for r in src]
    segs = {e: [] for e in range(E_l)}
    for tok, ids in rows:
        for j in range(8):
            e = int(ids[j]) - rank * E_l
            if 0 <= e < E_l:
                segs[e].append(tok * 8 + j)
    return segs
