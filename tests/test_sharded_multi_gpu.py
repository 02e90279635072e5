"""Sequence-sharded decode on real GPUs, one process per GPU (torchrun over
NCCL, 127.0.0.1): both exchange paths, bit-identical to each other and on
every rank, and checked against the oracle's sharded estimator (see
tests/mgpu_sharded_worker.py).  Skipped with fewer than two GPUs."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("world", [2, 4])
def test_sharded_decode_on_real_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(29600 + world), os.path.join(HERE, "mgpu_sharded_worker.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    out = res.stdout + res.stderr
    fails = "\n".join(line for line in out.splitlines() if " FAIL " in line)
    assert res.returncode == 0, (fails or out[-4000:])
    for r in range(world):
        assert f"RANK {r} OK" in out, (fails or out[-4000:])
