"""The folded expert-parallel exchange across two real GPUs (NVLink peer memory): runs tests/ep_exchange_worker.py
as two ranks under torch.distributed.run and requires both to report a bit-exact match with (layer, all-reduce)
per layer and oracle parity of the first layer. Skipped with fewer than two GPUs."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_two_rank_folded_exchange_matches_layer_allreduce():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29561",
           os.path.join(here, "ep_exchange_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    assert out.count("OK ") == 2, out[-3000:]
