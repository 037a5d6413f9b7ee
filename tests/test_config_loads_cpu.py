"""Host helpers of infer.net_b200/config_loads.py (the configs[3]/[4] measurement tool): its bf16
rounding equals the oracle's, and its per-GPU loads are the contiguous expert shards' route sums."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "infer.net_b200"))
import config_loads as CL  # noqa: E402
import oracle as O  # noqa: E402


def test_bf16_rounding_matches_oracle():
    rng = np.random.default_rng(1)
    a = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 10.0 ** rng.integers(-6, 6, 4096),
                        np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 1e-30, 3.3895314e38], np.float32)])
    assert np.array_equal(CL.bf16_bits(a), O.f32_to_bf16(a))


def test_loads_sum_contiguous_shards():
    rng = np.random.default_rng(2)
    ids = np.stack([rng.permutation(CL.E)[:8] for _ in range(300)]).astype(np.int32)
    ids[:40, 0] = np.arange(40) % 4  # skew toward the first shard
    r = CL.loads(ids)
    counts = np.bincount(ids.reshape(-1), minlength=CL.E)
    assert r["routes"] == ids.size
    for G in (2, 4, 8):
        per = [int(counts[g * CL.E // G:(g + 1) * CL.E // G].sum()) for g in range(G)]
        assert r[f"gpu_routes_G{G}"] == per
        assert abs(r[f"gpu_max_over_mean_G{G}"] - max(per) / np.mean(per)) < 1e-12
    assert abs(r["expert_max_over_mean"] - counts.max() / counts.mean()) < 1e-12
