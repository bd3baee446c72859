"""Expert parallelism on two GPUs: the peer-memory exchange (bs_ep_p2p_*) and
the NCCL all-to-all path must reproduce the single-GPU layer, over repeated
calls.  Runs tests/ep_gpu_worker.py as two torchrun ranks; skipped with fewer
than two GPUs."""

import os
import subprocess
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
@pytest.mark.multigpu
def test_expert_parallel_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(REPO, "tests", "ep_gpu_worker.py")]
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
