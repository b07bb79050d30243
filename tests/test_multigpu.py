"""Multi-GPU tests (one process per GPU, NCCL + NVLink peer memory). Skipped
when fewer than two GPUs are visible."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _torchrun(n, script, *args, timeout=420):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, DST_PG_TIMEOUT_S="120", NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={29400 + os.getpid() % 500}",
           os.path.join(ROOT, script), *args]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0


def test_fused_dp_adam_2gpu():
    _torchrun(2, "tests/suites/fused_dp_suite.py", "--dp", "2", "--device", "cuda", "--bf16")


def test_tp_suite_2gpu_nccl():
    _torchrun(2, "tests/suites/tp_suite.py", "--sp", "--vp", "--device", "cuda")


@pytest.mark.parametrize("sp", [True, False])
def test_tp_fused_2gpu(sp):
    _torchrun(2, "tests/suites/tp_fused_suite.py", *(["--sp"] if sp else []))
