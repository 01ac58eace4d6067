"""GPU-count invariance on real GPUs: the verify sweep under torchrun with 2 ranks
(NCCL over NVLink).  Column-parallel GEMM and head-parallel attention must give every
rank the single-GPU bits; skipped when fewer than 2 GPUs are visible."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_verify_across_two_gpus():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(
        [os.path.join(ROOT, "mlx-batch-invariant_b200"), ROOT, env.get("PYTHONPATH", "")])
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29533", "-m", "mlx_batch_invariant_b200", "verify", "--quick"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "GPU-count axis" in out and "all invariant" in out, out[-4000:]
    assert "VARIANT across GPU count" not in out
