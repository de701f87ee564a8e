"""Tensor-parallel (dense models) and expert-parallel (tiny-moe) decode on 2+
GPUs (one process per GPU, NCCL over NVLink): the sharded engine's argmax,
logits and greedy tokens equal the unsharded engine's and the oracle's.
Skipped on boxes with fewer GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _ngpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.parametrize("mode", ["peer-exchange", "nccl"])
@pytest.mark.parametrize("model,n", [("tiny-tp", 2), ("small-tp", 2), ("small-tp", 4), ("small-tp", 8),
                                     ("tiny-moe", 2), ("tiny-moe", 4)])
def test_tp_matches_single_gpu(model, n, mode):
    """peer-exchange: the residual partials go to every rank's memory from the
    GEMV epilogue and are summed in the next GEMV's prologue; nccl: the same
    sum through ncclAllReduce (INFERNO_TP_NCCL=1)."""
    if _ngpus() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", INFERNO_TP_NCCL="1" if mode == "nccl" else "0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", "--master-port=29517", str(ROOT / "tests" / "tp_worker.py"), model, "16"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "TP_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
