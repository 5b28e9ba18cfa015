"""Multi-GPU tests: real NVLink IPC peers, one process per GPU (torchrun children).

Skipped when fewer than 2 GPUs are visible.  NVLS is disabled for NCCL and the
kernels use plain peer loads/stores only.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(case, world, timeout=300):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), os.path.join(ROOT, "tests", "multigpu_worker.py"), "--case", case]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert proc.returncode == 0 and f"CASE-OK {case}" in proc.stdout, proc.stdout[-3000:] + proc.stderr[-5000:]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemm_rs_all_arms(world):
    _run("gemm_rs", world)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ag_gemm(world):
    _run("ag_gemm", world)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_model_matches_single_rank(world):
    _run("model", world)


@pytest.mark.parametrize("world", [2, 8])
def test_pull_scatter_matches_nccl(world):
    _run("scatter", world)


def test_missing_peer_times_out_cleanly():
    _run("missing_peer", 2)
