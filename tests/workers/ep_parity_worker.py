"""Worker of tests/test_gpu_ep.py (run under torchrun, one process per GPU).

Builds a small model twice -- full layers on every rank and the rank's expert shard -- runs the
expert-parallel stack on uneven contiguous token shards and compares the rows against the
single-GPU stack on all tokens. The same call is made twice (the second must repeat the first bit
for bit: the peer buffers' arrival counters carry over between calls), then once with three times
the tokens (every rank grows and re-maps its peer buffers); then one layer of a 256-expert
model, whose router runs on the tensor cores with the exact candidate check, and one layer of the
full geometry (D 2048, 256 experts, I 512) with 1024 tokens per rank. (One layer: deeper layers
see inputs that differ in the last bits -- the ranks' partial rows are summed in another order
than the single-GPU combine -- and with 256 experts a near-tie can then route a token
differently, which is not a fault.)

Routing is checked at every layer of every case: the expert-parallel stack dumps each layer's
input rows and expert ids on this rank; the ids must equal, bit for bit, those of the single-GPU
block with every router logit in the canonical order (DI_MOE_ROUTER_EXACT) on the same rows, and
those of the CPU oracle on sampled rows. Exits non-zero on a mismatch.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "infer.net_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import deepinfer_cuda as di  # noqa: E402
import oracle as O  # noqa: E402

rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
local = int(os.environ.get("LOCAL_RANK", rank))
torch.cuda.set_device(local)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
E, D, I, L, SEED = 64, 256, 128, 3, 77
bits = int(os.environ.get("EP_BITS", "8"))
sizes = [40 + 16 * r for r in range(world)]  # uneven shards, in rank order
T = sum(sizes)
ctx = di.Context(resident=0)
uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
if rank == 0:
    uid.copy_(torch.frombuffer(bytearray(di.ExpertParallel.unique_id()), dtype=torch.uint8))
dist.broadcast(uid, 0)
ep = di.ExpertParallel(ctx, bytes(uid.cpu().numpy().tobytes()), rank, world)
shards = [ep.layer(di.generate_layer_matrices(ctx, SEED, l, bits, E, D, I, shard=(rank, world))) for l in range(L)]
full = [di.MoeLayer(ctx, di.generate_layer_matrices(ctx, SEED, l, bits, E, D, I)) for l in range(L)]
rng = np.random.default_rng(5)  # the same inputs on every rank
pick = np.random.default_rng(100 + rank)  # this rank's sampled rows
norms = (1.0 + 0.1 * np.cos(np.arange(L * D))).astype(np.float32).reshape(L, D)


def routes_ok(ht, it, seed, bits):
    """Every layer's ids on this rank against the all-exact single-GPU router on the same rows, and
    sampled rows against the CPU oracle."""
    ok = True
    for l in range(ht.shape[0]):
        _, ids, _, _ = di.moe_block(full[l], ht[l], di.PATH_GROUPED | di.ROUTER_EXACT)
        ok = ok and np.array_equal(ids, it[l])
        rows = np.sort(pick.choice(ht.shape[1], min(4, ht.shape[1]), replace=False))
        rc, _, oids, _, _ = O.moe_block(O.Layer(seed, layer=l, bits=bits, E=E, D=D, I=I), ht[l][rows], O.MODE_F32)
        ok = ok and rc == 0 and np.array_equal(oids, it[l][rows])
    return ok


def check(sizes, label, seed, previous=None):
    T = sum(sizes)
    x = rng.standard_normal((T, D)).astype(np.float32) if previous is None else previous[0]
    lo = sum(sizes[:rank])
    xs = x[lo:lo + sizes[rank]].copy()
    n = len(shards)
    ht = np.zeros((n, sizes[rank], D), np.uint16)
    it = np.zeros((n, sizes[rank], 8), np.int32)
    ep.stack(shards, norms, xs, sizes[rank], 1e-6, 0, h_trace=ht, ids_trace=it)
    ref, _, _, _ = di.moe_stack(ctx, full, norms, x, 1e-6, di.PATH_GROUPED)
    ref = ref[lo:lo + sizes[rank]]
    err = np.abs(xs.astype(np.float64) - ref)
    rel = np.linalg.norm(xs - ref) / np.linalg.norm(ref)
    ok = float(err.max()) <= 2e-2 and rel <= 5e-3
    rok = routes_ok(ht, it, seed, bits)
    if previous is not None:
        ok = ok and np.array_equal(xs, previous[1])
    print(f"rank {rank} {label}: rows {sizes[rank]} max_abs {err.max():.3e} rel_l2 {rel:.3e} routes {rok} ok {ok}",
          flush=True)
    return ok and rok, (x, xs)


ok1, first = check(sizes, "first", SEED)
ok2, _ = check(sizes, "repeat", SEED, previous=first)
ok3, _ = check([3 * n for n in sizes], "grown", SEED)
for l in shards + full:
    l.close()
# the full expert count: 256 experts, hidden 512, intermediate 512 (the tensor-core router), then
# the full geometry
oks = []
for E, D, I, L, seed, per_rank in ((256, 512, 512, 1, SEED + 1, None), (256, 2048, 512, 1, SEED + 2, 1024)):
    shards = [ep.layer(di.generate_layer_matrices(ctx, seed, l, bits, E, D, I, shard=(rank, world))) for l in range(L)]
    full = [di.MoeLayer(ctx, di.generate_layer_matrices(ctx, seed, l, bits, E, D, I)) for l in range(L)]
    norms = (1.0 + 0.1 * np.cos(np.arange(L * D))).astype(np.float32).reshape(L, D)
    case = [4 * n for n in sizes] if per_rank is None else [per_rank] * world
    oks.append(check(case, f"{E} experts, hidden {D}", seed)[0])
    for l in shards + full:
        l.close()
    shards, full = [], []
ok = ok1 and ok2 and ok3 and all(oks)
flag = torch.tensor([0 if ok else 1], device="cuda")
dist.all_reduce(flag)
for l in shards + full:
    l.close()
ep.close()
ctx.close()
dist.destroy_process_group()
sys.exit(int(flag.item() != 0))
