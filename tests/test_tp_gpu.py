"""Tensor parallel on real GPUs: NCCL and fused (NVSwitch multimem) paths vs TP=1; bounded peer waits."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_peer_barrier_times_out_with_status():
    """A barrier whose peer never announces gives up within its budget and reports kErrPeerWait.

    Single GPU, no peer memory: both pad pointers address this rank's own pad,
    and slot 1 (the "peer") is never written.
    """
    if not torch.cuda.is_available():
        pytest.skip("no CUDA")
    from granite_switch_b200._native import ERR_PEER_WAIT, err_buffer, native, read_errors

    dev = torch.device("cuda", 0)
    err_buffer(dev)
    read_errors(dev)
    pad = torch.zeros(64, dtype=torch.int32, device=dev)
    ptrs = torch.tensor([pad.data_ptr(), pad.data_ptr()], dtype=torch.int64, device=dev)
    ctr = torch.zeros(1, dtype=torch.int32, device=dev)  # epoch 1 is announced, never answered
    native().peer_barrier(ptrs, 0, 2, ctr, 200_000_000, err_buffer(dev))  # 0.2 s budget
    torch.cuda.synchronize()
    assert read_errors(dev) & ERR_PEER_WAIT
    assert int(ctr.item()) == 1  # the device counter advanced
    # the context stays usable
    x = torch.ones(4, device=dev)
    assert float(x.sum()) == 4.0


@pytest.mark.multigpu
def test_tp2_matches_tp1():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531", "-m",
           "granite_switch_b200.parallel.tp_check", "--engine"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0, r.stderr[-2000:]
    assert '"mode": "nccl"' in r.stdout
    assert '"mode": "engine_async_vs_sync"' in r.stdout


@pytest.mark.multigpu
def test_pp2_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29535", "-m",
           "granite_switch_b200.parallel.pp_check"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0, r.stderr[-2000:]
    assert '"ok": true' in r.stdout
