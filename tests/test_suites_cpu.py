"""The five correctness suites as multi-process gloo runs on CPU.

Flag combinations follow the reference README's matrix (``README.md:164-169``)
plus the compositions the reference could not run on NCCL (interleaved x TP).
"""

import os
import sys

import pytest

from dstraining_b200.utils.launch import launch

SUITES = os.path.join(os.path.dirname(__file__), "suites")


def run(n, script, *args, timeout=540):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    assert launch(n, [os.path.join(SUITES, script), "--device", "cpu", *args], timeout=timeout, env=env) == 0


@pytest.mark.parametrize("args", [(), ("--sp",), ("--sp", "--recompute", "--vp"), ("--vp",)])
def test_tp_suite(args):
    run(2, "tp_suite.py", *args)


def test_tp4_sp_vp():
    run(4, "tp_suite.py", "--sp", "--vp")


@pytest.mark.parametrize(
    "n,args",
    [
        (2, ("--pp", "2")),
        (4, ("--pp", "4", "--micro", "1")),
        (4, ("--pp", "2", "--tp", "2", "--sp")),
        (4, ("--pp", "2", "--tp", "2", "--chunks", "2", "--micro", "1", "--sp")),
        (2, ("--pp", "2", "--chunks", "2", "--micro", "1")),
    ],
)
def test_pp_suite(n, args):
    run(n, "pp_suite.py", *args)


@pytest.mark.parametrize(
    "n,args",
    [
        (2, ("--dp", "2")),
        (2, ("--dp", "2", "--bucketed")),
        (4, ("--dp", "2", "--tp", "2", "--sp", "--bucketed")),
        (4, ("--dp", "2", "--pp", "2", "--micro", "1", "--bucketed")),
        (8, ("--dp", "2", "--pp", "2", "--tp", "2", "--chunks", "2", "--micro", "1", "--sp", "--bucketed")),
    ],
)
def test_dp_suite(n, args):
    run(n, "dp_suite.py", *args)


def test_precision_suite():
    run(2, "precision_suite.py")


def test_recompute_suite():
    import subprocess

    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, os.path.join(SUITES, "recompute_suite.py")], env=env, timeout=300)
    assert r.returncode == 0
