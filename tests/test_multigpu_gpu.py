"""Multi-GPU paths over NCCL on one box: context-parallel split-KV (config 4) and row sharding
(config 5). Runs ``mp_nccl_worker.py`` under torchrun with one rank per GPU (two ranks, or
``PD_TEST_RANKS``); skipped on a host with fewer GPUs than that.

The ranks never wait on each other inside a kernel: partials cross GPUs only through one NCCL
all-gather into local memory. The process group has a 60 s timeout and the whole launch is
bounded by ``timeout -k 30``, so a rank that fails ends the test instead of holding the GPUs.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_context_parallel_and_row_sharding_over_nccl(tmp_path):
    ranks = int(os.environ.get("PD_TEST_RANKS", "2"))
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs, found {torch.cuda.device_count()}")
    summary = tmp_path / "summary.json"
    cmd = ["timeout", "-k", "30", "420", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={ranks}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(HERE / "mp_nccl_worker.py"), str(summary)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=480)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    result = json.loads(summary.read_text())
    assert result["passed"] and result["world"] == ranks
    assert result["cp_identical_on_all_ranks"]
    assert result["rows_total"] == 1024
