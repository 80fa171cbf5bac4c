"""Fold-CP across real GPUs: one process per GPU (torch.distributed.run, NCCL), both band
transports, against the single-device stack. Runs on boxes with at least two GPUs."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("gpus,mesh", [(2, "1x2"), (4, "2x2"), (8, "2x4")])
def test_cp_processes_match_single_device(gpus, mesh):
    if torch.cuda.device_count() < gpus:
        pytest.skip(f"needs {gpus} GPUs")
    env = dict(os.environ, OPENDDE_FOLDCP_MESH=mesh, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={gpus}", "--master-addr=127.0.0.1", "--master-port=29571",
           os.path.join(HERE, "foldcp_mp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "OK" in r.stdout
