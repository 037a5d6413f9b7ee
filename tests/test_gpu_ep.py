"""Expert parallelism on 2 and 8 GPUs (di_moe_ep_stack) against the single-GPU stack and the oracle.

Runs tests/workers/ep_parity_worker.py under torchrun with one process per GPU; each case needs
as many GPUs as it has ranks and is skipped otherwise.
"""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ranks", [2, 8])
@pytest.mark.parametrize("bits", [8, 5])
def test_expert_parallel_matches_single_gpu(bits, ranks):
    import torch
    n = torch.cuda.device_count()
    if n < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    env = dict(os.environ, EP_BITS=str(bits), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(ranks), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "workers", "ep_parity_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
