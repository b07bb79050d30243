"""API compatibility: the reference's own five correctness scripts, unmodified,
run against this framework's ``dst`` package on gloo ranks (CPU).

The scripts come from the reference installed under ``baseline/_ref``; they
are copied to a temporary directory so that ``import dst`` resolves to this
repository's package instead of the reference's. Flags follow the
reference's quick-start matrix (``README.md:164-169``). Skipped when the
reference is not installed."""

import os
import shutil
import sys

import pytest

from dstraining_b200.utils.launch import launch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_TESTS = os.path.join(ROOT, "baseline", "_ref", "tests")

pytestmark = pytest.mark.skipif(not os.path.isdir(REF_TESTS), reason="reference not installed under baseline/_ref")


@pytest.fixture(scope="module")
def suites(tmp_path_factory):
    d = tmp_path_factory.mktemp("refcompat")
    shutil.copytree(REF_TESTS, d / "tests")
    return d / "tests"


def _env():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    return env


@pytest.mark.parametrize(
    "n,script,args",
    [
        (2, "test_tp_correctness.py", ("--sp", "--recompute", "--vp")),
        (4, "test_pp_correctness.py", ("--pp", "2", "--tp", "2", "--chunks", "2", "--micro", "1", "--sp")),
        (8, "test_dp_correctness.py", ("--dp", "2", "--pp", "2", "--tp", "2", "--chunks", "2", "--micro", "1",
                                       "--sp", "--bucketed")),
        (2, "test_precision.py", ()),
        (1, "test_recompute.py", ()),
    ],
)
def test_reference_suite_passes_on_our_dst(suites, n, script, args):
    path = str(suites / script)
    assert launch(n, [path, *args], timeout=600, env=_env()) == 0, script


def test_dst_resolves_to_this_repository(suites):
    import subprocess

    out = subprocess.run([sys.executable, "-c", "import dst, os; print(os.path.dirname(dst.__file__))"],
                         cwd=str(suites), env=_env(), capture_output=True, text=True, check=True).stdout.strip()
    assert os.path.realpath(out) == os.path.realpath(os.path.join(ROOT, "dst"))


def test_reference_train_script_runs_on_our_dst(tmp_path):
    """The reference's train.py (copied next to nothing else, so ``dst`` is
    this repository's) with every axis at once, as in its quick start."""
    src = os.path.join(ROOT, "baseline", "_ref", "train.py")
    if not os.path.exists(src):
        pytest.skip("reference not installed under baseline/_ref")
    shutil.copy(src, tmp_path / "train.py")
    args = ["--dp", "2", "--tp", "2", "--pp", "2", "--chunks", "2", "--sp", "--vp", "--recompute", "--bf16",
            "--micro", "2", "--steps", "4", "--data", "synthetic", "--device", "cpu"]
    assert launch(8, [str(tmp_path / "train.py"), *args], timeout=600, env=_env()) == 0


def test_every_public_name_of_the_reference_modules():
    """Each name a reference ``dst`` module defines at top level (functions,
    classes, constants; plus ``_Recompute``, which its tests patch) exists in
    the module of the same name here. Read from the reference's source as
    text (AST), so nothing of it is imported."""
    import ast
    import importlib

    ref_pkg = os.path.join(ROOT, "baseline", "_ref", "dst")
    missing = []
    for fname in sorted(os.listdir(ref_pkg)):
        if not fname.endswith(".py") or fname == "__init__.py":
            continue
        with open(os.path.join(ref_pkg, fname)) as f:
            tree = ast.parse(f.read())
        names = set()
        for node in tree.body:
            if isinstance(node, (ast.FunctionDef, ast.ClassDef)):
                names.add(node.name)
            elif isinstance(node, ast.Assign):
                names.update(t.id for t in node.targets if isinstance(t, ast.Name))
        public = {n for n in names if not n.startswith("_")} | ({"_Recompute"} & names)
        ours = importlib.import_module(f"dst.{fname[:-3]}")
        missing += [f"dst.{fname[:-3]}.{n}" for n in sorted(public) if not hasattr(ours, n)]
    assert not missing, missing
