"""Expert parallelism across real GPUs: tests/ep_worker.py under torchrun on
2 (and up to 8) GPUs of one box, each rank's output bitwise equal to a
single-GPU plan's on the same rows. Skipped on a box with one GPU (the
one-GPU local-group tests cover the same data path)."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,placement,rows", [(2, "contiguous", 4096), (2, "strided", 1000),
                                                  (2, "balanced", 4096), (4, "contiguous", 8192),
                                                  (4, "balanced", 8192), (8, "contiguous", 32768),
                                                  (8, "balanced", 32768)])
def test_ep_ranks_equal_single_gpu(world, placement, rows):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, EP_STRIDED="1" if placement == "strided" else "0",
               EP_BALANCED="1" if placement == "balanced" else "0", EP_ROWS=str(rows), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "ep_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(r.stdout[-2000:], r.stderr[-4000:])
    assert r.returncode == 0
    assert "EP_OK" in r.stdout


def test_ep_missing_peer_times_out():
    """A rank that never joins a forward: the others' bounded device barrier
    gives up after UOCR_EP_WAIT_MS (1 s here) and check() reports a timeout."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, EP_MODE="timeout", EP_ROWS="1024", UOCR_EP_WAIT_MS="1000", NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "ep_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(r.stdout[-2000:], r.stderr[-4000:])
    assert r.returncode == 0
    assert "EP_TIMEOUT_OK" in r.stdout
