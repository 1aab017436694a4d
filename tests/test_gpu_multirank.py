"""Two ranks over NCCL (libljx's halo) against the CPU oracle on one crystal.

Launches tests/multirank_parity.py under torchrun, one rank per GPU, on boxes with two GPUs or
more: every owned force (matched by global site id), the collective energy and virial of both
exchange patterns (C3's forward F', C4's reverse rho / forward F' / reverse forces) must match
the oracle's evaluation of the whole periodic crystal. Skipped on one-GPU boxes, where
tests/test_gpu_halo.py covers the same library code with a one-rank communicator.
"""

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_rank_decomposition_matches_oracle(tmp_path):
    out = tmp_path / "multirank.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(free_port()), str(ROOT / "tests" / "multirank_parity.py"),
           "--out", str(out)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    summary = json.loads(out.read_text())
    assert summary["pass"] and summary["ranks"] == 2
    for mode in ("rows-full", "half-unique", "rows-full+overlap", "half-unique+overlap"):
        m = summary["modes"][mode]
        assert m["pass"], m
