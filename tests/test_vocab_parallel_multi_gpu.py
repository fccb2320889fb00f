"""Vocabulary-parallel sampling over real ranks: one process per GPU, NCCL all-gather over NVLink.

Runs tests/vp_dist_worker.py under torchrun on 2, 4 and 8 GPUs (each skipped on a box with fewer),
with NVLS off.
"""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_ranks_match_full_rows(ranks):
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={ranks}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(REPO, "tests", "vp_dist_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert f"vocab-parallel OK on {ranks} GPUs" in r.stdout
