"""Multi-GPU checks, each run as one process per GPU under torch.distributed
(skipped when fewer than 2 GPUs are visible): the gathered norm of
gdn_chunked_norm_gather_ws against the single-GPU path
(tests/mgpu/norm_gather_check.py), and the whole layer on head shards against
the layer on one GPU (tests/mgpu/layer_check.py)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(script):
    cnt = torch.cuda.device_count()
    n = 8 if cnt >= 8 else (4 if cnt >= 4 else 2)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "mgpu", script)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    return subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_norm_gather_over_nvlink_matches_single_gpu():
    r = run_ranks("norm_gather_check.py")
    assert r.returncode == 0, r.stdout[:4000] + "\n...\n" + r.stdout[-2000:] + r.stderr[:6000]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_layer_matches_single_gpu_layer():
    r = run_ranks("layer_check.py")
    assert r.returncode == 0, r.stdout[:4000] + "\n...\n" + r.stdout[-2000:] + r.stderr[:6000]
