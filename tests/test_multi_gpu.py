"""Vocab-sharded sampling over real NCCL ranks (one process per GPU).

Runs tests/mgpu_worker.py under torch.distributed.run on 2 GPUs (skipped
with fewer), through the library's own communicator
(verbo_cuda_sharded_sample: one NCCL all-gather of packed candidates): the
sharded ids must equal the C oracle's on the full rows (away from boundaries)
and agree on every rank, for column shards of logits rows and for the
tensor-parallel logits tail (vocab shards of the LM head) against the
oracle's tail.  The CPU tests of the same host logic (gloo) are in
tests/test_distributed.py.
"""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_vocab_sharded_over_two_gpus_matches_oracle(cuda_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           str(ROOT / "tests" / "mgpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "== oracle: True" in r.stdout
    assert "== oracle tail + pick: True" in r.stdout
