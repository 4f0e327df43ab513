"""Sequence-parallel BSA on 2 GPUs (torchrun, NCCL): both exchanges (copy engines, messages) return
exactly the single-GPU result.  Skipped where fewer than 2 GPUs are visible."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ulysses_two_gpus_equals_single_gpu():
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29517",
           os.path.join(HERE, "_ulysses_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0 and "ULYSSES_PARITY_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])
