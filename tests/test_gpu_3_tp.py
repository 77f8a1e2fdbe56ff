"""Tensor parallelism on 2 GPUs: Engine(tp=2) over NCCL gives the single-GPU greedy tokens, every rank the same
tokens, and CUDA-graph replay the same tokens as eager steps. Skipped with fewer than 2 GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["small-1k", "small"])
def test_tp2_matches_single_gpu(name):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "tp_worker.py"), name]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("[")][-1]
    ranks = json.loads(line)
    assert all(x["status"] == 0 for x in ranks)
    assert all(x["ar_exact"] in (True, None) for x in ranks)  # None: no symmetric memory, NCCL carried the sums
    assert ranks[0]["greedy"] == ranks[1]["greedy"] == ranks[0]["eager"] == ranks[1]["eager"]
    assert ranks[0]["sample"] == ranks[1]["sample"]
    assert ranks[0]["greedy"] == ranks[0]["ref_greedy"]
