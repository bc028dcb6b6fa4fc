"""Sharded decode on 2+ GPUs (NCCL over NVLink): runs tests/sharded_worker.py under torchrun.
Skipped when fewer than two GPUs are visible (the round-end GPU suite runs on one)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")
def test_seq_and_head_sharded_decode_match_single_gpu():
    world = min(torch.cuda.device_count(), 8)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "sharded_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    print(res.stdout[-4000:], res.stderr[:6000], res.stderr[-1500:])
    assert res.returncode == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")
def test_tensor_parallel_decoder_matches_the_sdpa_forward():
    """TPDecoder on every visible GPU (up to the 8 KV heads' worth) against HF's SDPA forward over the
    same spliced cache (tests/tp_worker.py)."""
    world = min(torch.cuda.device_count(), 8)
    world = max(w for w in (1, 2, 4, 8) if w <= world)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "tp_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    print(res.stdout[-4000:], res.stderr[:6000], res.stderr[-1500:])
    assert res.returncode == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")
def test_peer_memory_sums_match_the_collective_library():
    """threadcut_b200.peer.AllReduce (tests/peer_worker.py) on every visible GPU (up to 8)."""
    world = max(w for w in (2, 4, 8) if w <= min(torch.cuda.device_count(), 8))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "peer_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    print(res.stdout[-4000:], res.stderr[:6000], res.stderr[-1500:])
    assert res.returncode == 0
