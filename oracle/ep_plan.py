"""Expert-parallel dispatch plan restated in numpy (TEST INFRASTRUCTURE ONLY).

Mirrors the bookkeeping of infer.net_b200/csrc/ep.cuh so that the multi-rank logic can be
checked on CPU ranks: a token is sent once to every rank that owns one of its experts, in
its row slot is its local token index in every destination; a receiver orders the routes of each of its experts by
(source rank, source row, slot). The claim checked by tests/test_ep_plan_cpu.py: with token
shards contiguous in rank order, this equals the single-GPU stable permutation
(native/DeepInfer.Metal/prefill_moe.mm:12-14 order) restricted to the rank's experts.
"""
import numpy as np


def layout(ids: np.ndarray, E_l: int, G: int):
    """sent [T, G]: whether token t's row goes to rank d (d owns one of t's experts). Rows are not
    compacted: token t occupies row slot t of its source region in every destination."""
    T = ids.shape[0]
    sent = np.zeros((T, G), bool)
    for t in range(T):
        sent[t, sorted(set((ids[t] // E_l).tolist()))] = True
    return sent


def pack(ids: np.ndarray, tok0: int, E_l: int, G: int):
    """Row slots for each destination: (global token, 8 ids, sent) for every local token, in
    token order (the metadata of every slot is written; the row data only where sent)."""
    sent = layout(ids, E_l, G)
    rows = [[(tok0 + t, ids[t].copy(), bool(sent[t, d])) for t in range(ids.shape[0])] for d in range(G)]
    return rows, sent


def receive_permutation(recv_rows_by_source, rank: int, E_l: int):
    """Concatenate row slots in source-rank order; stable-sort the local routes by local expert.
    Returns {local expert: [global route ids]}. A slot with a local route must have been sent."""
    rows = [r for src in recv_rows_by_source for r in src]
    segs = {e: [] for e in range(E_l)}
    for tok, ids, sent in rows:
        for j in range(8):
            e = int(ids[j]) - rank * E_l
            if 0 <= e < E_l:
                if not sent:
                    raise AssertionError(f"token {tok} has a route on rank {rank} but was not sent there")
                segs[e].append(tok * 8 + j)
    return segs
