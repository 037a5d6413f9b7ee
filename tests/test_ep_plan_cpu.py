"""Expert-parallel dispatch plan on two CPU (gloo) ranks.

Each rank routes its contiguous token shard, sends one row per (token, destination rank), and
builds the expert-grouped permutation of what it receives; the result must equal the
single-GPU stable permutation restricted to the rank's experts, and every token's partial
rows must come back to it (combine bookkeeping).
"""
import os
import socket

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

import ep_plan
import oracle as O


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _global_ids(T, E, seed):
    rng = np.random.default_rng(seed)
    return np.stack([rng.permutation(E)[:8] for _ in range(T)]).astype(np.int32)


def _worker(rank, world, port, T, E, sizes, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids = _global_ids(T, E, 3)
        E_l = E // world
        lo = sum(sizes[:rank])
        rows, sent = ep_plan.pack(ids[lo:lo + sizes[rank]], lo, E_l, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, rows)
        received = [gathered[src][rank] for src in range(world)]
        segs = ep_plan.receive_permutation(received, rank, E_l)
        counts, offsets, routes = O.permute(ids, E)
        ok = all(segs[e] == routes[offsets[rank * E_l + e]:offsets[rank * E_l + e] + counts[rank * E_l + e]].tolist()
                 for e in range(E_l))
        # combine bookkeeping: each (token, destination) pair maps to exactly one returned row
        for t in range(sizes[rank]):
            dests = sorted(set((ids[lo + t] // E_l).tolist()))
            ok &= [d for d in range(world) if sent[t, d]] == dests
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_dispatch_plan_matches_global_permutation():
    world, T, E = 2, 150, 64
    sizes = [61, 89]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, E, sizes, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert results == {0: True, 1: True}


def test_single_rank_plan_is_identity():
    ids = _global_ids(33, 32, 4)
    rows, _ = ep_plan.pack(ids, 0, 32, 1)
    segs = ep_plan.receive_permutation([rows[0]], 0, 32)
    counts, offsets, routes = O.permute(ids, 32)
    assert all(segs[e] == routes[offsets[e]:offsets[e] + counts[e]].tolist() for e in range(32))


def test_rows_sent_to_extra_ranks_are_ignored():
    # the router stores a token's row into every rank that owns one of its CANDIDATE experts before
    # the exact top-8 is known; a rank that owns none of the final 8 receives the row but no route
    E, G, T = 64, 4, 97
    E_l = E // G
    ids = _global_ids(T, E, 5)
    counts, offsets, routes = O.permute(ids, E)
    rng = np.random.default_rng(6)
    rows, sent = ep_plan.pack(ids, 0, E_l, G)
    extra = rng.random((T, G)) < 0.3
    for d in range(G):
        rows[d] = [(tok, i, s or bool(extra[tok, d])) for tok, i, s in rows[d]]
    for r in range(G):
        segs = ep_plan.receive_permutation([rows[r]], r, E_l)
        assert all(segs[e] == routes[offsets[r * E_l + e]:offsets[r * E_l + e] + counts[r * E_l + e]].tolist()
                   for e in range(E_l))
