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


@pytest.mark.parametrize("args", [(), ("--sp",), ("--sp", "--recompute", "--vp"), ("--vp",),
                                  ("--sp", "--recompute-blocks", "--vp")])
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


@pytest.mark.parametrize("n,args", [(2, ("--tp", "2")), (4, ("--tp", "2", "--pp", "2")),
                                    (4, ("--tp", "2", "--pp", "2", "--background"))])
def test_checkpoint_suite(n, args, tmp_path):
    run(n, "ckpt_suite.py", *args, "--dir", str(tmp_path / "ckpt"))


def test_train_cli_all_axes_and_resume(tmp_path):
    """train.py with dp x pp x tp x interleaving x SP on 8 gloo ranks, then a
    resume from its checkpoint."""
    root = os.path.dirname(SUITES)
    train = os.path.join(os.path.dirname(root), "train.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    ck = str(tmp_path / "ck")
    common = ["--dp", "2", "--pp", "2", "--tp", "2", "--chunks", "2", "--sp", "--recompute", "--vp",
              "--micro", "1", "--batch", "4", "--device", "cpu", "--ckpt-dir", ck, "--jsonl", str(tmp_path / "m.jsonl"),
              "--heartbeat-timeout", "120"]  # healthy job: the watchdog must not fire
    assert launch(8, [train, "--steps", "4", "--ckpt-every", "2", "--ckpt-async", *common], timeout=540, env=env) == 0
    assert sorted(os.listdir(ck)) == ["step_00000002", "step_00000004"]
    assert all(os.path.exists(os.path.join(ck, d, "COMPLETE")) for d in os.listdir(ck))
    assert launch(8, [train, "--steps", "6", "--resume", *common], timeout=540, env=env) == 0
    lines = (tmp_path / "m.jsonl").read_text().splitlines()
    assert len(lines) == 6  # steps 0-3, then 4-5 after the resume
    import json

    rec = json.loads(lines[-1])
    assert rec["step"] == 5 and rec["status"] == 0 and rec["step_ms_max"] > 0 and rec["tok_s"] > 0


@pytest.mark.parametrize("n,args", [(2, ("--dp", "2")), (4, ("--dp", "2", "--tp", "2", "--sp")), (4, ("--dp", "4",)),
                                    (4, ("--dp", "4", "--transport", "collectives")),
                                    (4, ("--dp", "2", "--tp", "2", "--sp", "--transport", "collectives"))])
def test_fused_dp_suite(n, args):
    run(n, "fused_dp_suite.py", *args)


@pytest.mark.parametrize("mode", ["raise", "hang", "exit"])
def test_failure_detection(mode, tmp_path):
    """A rank fails on the host (raises, hangs, or exits); the job must end
    with a non-zero status long before the process-group timeout, with the
    survivors' watchdogs reporting the failure."""
    import time

    marker = str(tmp_path / "m")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    t0 = time.time()
    rc = launch(3, [os.path.join(SUITES, "fault_suite.py"), "--mode", mode, "--victim", "1", "--marker", marker],
                timeout=120, env=env)
    assert rc != 0
    assert time.time() - t0 < 60
    assert any(os.path.exists(f"{marker}.{r}") for r in range(3)), "no rank detected the failure"


def test_step_gate_detects_departed_rank(tmp_path):
    """A rank exits cleanly between steps; the survivor's step gate raises
    before the next step launches anything."""
    import time

    marker = str(tmp_path / "g")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    t0 = time.time()
    rc = launch(2, [os.path.join(SUITES, "gate_suite.py"), "--marker", marker], timeout=120, env=env)
    assert rc != 0
    assert time.time() - t0 < 60
    with open(f"{marker}.0") as f:
        assert f.read().startswith("4 ")  # rank 0 noticed at step 4


@pytest.mark.parametrize("n", [1, 2])
def test_grad_accumulation(n):
    run(n, "accum_suite.py")


def test_restart_from_checkpoint(tmp_path):
    """A rank fails at step 3 (host-side injection, once); the launcher stops
    the job and relaunches it with --resume; training continues from the step-2
    checkpoint and ends bitwise identical to an uninterrupted run."""
    import torch

    from dstraining_b200.utils.launch import launch_with_restarts

    root = os.path.dirname(SUITES)
    train = os.path.join(os.path.dirname(root), "train.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    common = ["--dp", "2", "--layers", "2", "--heads", "4", "--embd", "64", "--block", "32", "--vocab", "256",
              "--batch", "4", "--steps", "6", "--ckpt-every", "2", "--device", "cpu"]
    assert launch(2, [train, *common, "--ckpt-dir", str(tmp_path / "ref")], timeout=300, env=env) == 0
    once = tmp_path / "injected"
    fenv = dict(env, DST_INJECT_FAULT="1:3", DST_INJECT_FAULT_ONCE=str(once))
    rc = launch_with_restarts(2, [train, *common, "--ckpt-dir", str(tmp_path / "ck")], max_restarts=1,
                              restart_args=["--resume"], timeout=300, env=fenv)
    assert rc == 0 and once.exists()
    a = torch.load(tmp_path / "ref" / "step_00000006" / "shard_tp0_pp0.pt")
    b = torch.load(tmp_path / "ck" / "step_00000006" / "shard_tp0_pp0.pt")
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)


def test_block_recompute_single_process():
    """Full-block recompute: bitwise-identical loss and gradients, fewer bytes
    saved for backward."""
    import torch

    from dstraining_b200.models.gpt import GPT, GPTConfig
    from dstraining_b200.parallel.topology import SINGLE

    cfg = GPTConfig(vocab_size=256, block_size=32, n_layer=3, n_head=4, n_embd=64)
    idx = torch.randint(0, 256, (4, 32), generator=torch.Generator().manual_seed(0))

    def run(flag):
        m = GPT(GPTConfig(**{**vars(cfg), "recompute_blocks": flag}), SINGLE, seed=1)
        saved = [0]

        def pack(t):
            saved[0] += t.numel() * t.element_size()
            return t

        with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
            _, loss = m(idx, idx)
        loss.backward()
        return loss, {n: p.grad for n, p in m.named_parameters()}, saved[0]

    l0, g0, b0 = run(False)
    l1, g1, b1 = run(True)
    assert torch.equal(l0, l1)
    assert all(torch.equal(g0[n], g1[n]) for n in g0)
    assert b1 < b0 / 2, (b0, b1)


def test_eval_matches_across_pipeline_layouts(tmp_path):
    """--eval-every: held-out loss after 2 training steps is the same whether
    the model runs in one piece, as a 1F1B pipeline or as an interleaved
    pipeline (forward-only schedules)."""
    import json

    root = os.path.dirname(SUITES)
    train = os.path.join(os.path.dirname(root), "train.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    common = ["--layers", "4", "--heads", "4", "--embd", "64", "--block", "32", "--vocab", "256", "--batch", "4",
              "--micro", "2", "--steps", "2", "--eval-every", "2", "--eval-batches", "2", "--device", "cpu"]
    out = {}
    for name, n, extra in [("single", 1, []), ("1f1b", 2, ["--pp", "2"]), ("interleaved", 2, ["--pp", "2", "--chunks", "2"])]:
        sink = tmp_path / f"{name}.jsonl"
        assert launch(n, [train, *common, *extra, "--jsonl", str(sink)], timeout=300, env=env) == 0, name
        evals = [json.loads(ln)["eval_loss"] for ln in sink.read_text().splitlines() if "eval_loss" in ln]
        assert len(evals) == 1, name
        out[name] = evals[0]
    assert abs(out["single"] - out["1f1b"]) < 1e-4 and abs(out["single"] - out["interleaved"]) < 1e-4, out


def test_elastic_restart_on_fewer_ranks(tmp_path):
    """tp2 x dp2 on 4 ranks; a rank fails at step 3; the job comes back on 2
    ranks as tp1 x dp2 from the resharded step-2 checkpoint and finishes with
    weights matching an uninterrupted tp2 run (fp32, up to rounding)."""
    import torch

    from dstraining_b200.models.gpt import GPT, GPTConfig
    from dstraining_b200.parallel.topology import SINGLE
    from dstraining_b200.utils import checkpoint
    from dstraining_b200.utils.launch import launch_with_restarts

    root = os.path.dirname(SUITES)
    train = os.path.join(os.path.dirname(root), "train.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    common = ["--dp", "2", "--tp", "2", "--layers", "2", "--heads", "4", "--embd", "64", "--block", "32",
              "--vocab", "256", "--batch", "4", "--steps", "6", "--ckpt-every", "2", "--device", "cpu"]
    assert launch(4, [train, *common, "--ckpt-dir", str(tmp_path / "ref")], timeout=300, env=env) == 0
    once = tmp_path / "injected"
    fenv = dict(env, DST_INJECT_FAULT="1:3", DST_INJECT_FAULT_ONCE=str(once))
    rc = launch_with_restarts(4, [train, *common, "--ckpt-dir", str(tmp_path / "ck")], max_restarts=1,
                              restart_args=["--resume", "--tp", "1"], timeout=300, env=fenv, restart_nproc=2)
    assert rc == 0 and once.exists()
    info = checkpoint.inspect(str(tmp_path / "ck" / "step_00000006"))
    assert info["ok"] and info["topology"]["tp"] == 1

    def full(path):
        m = GPT(GPTConfig(vocab_size=256, block_size=32, n_layer=2, n_head=4, n_embd=64), SINGLE, seed=0)
        checkpoint.load(path, m, None, SINGLE)
        return dict(m.named_parameters())

    a, b = full(str(tmp_path / "ref" / "step_00000006")), full(str(tmp_path / "ck" / "step_00000006"))
    assert max((a[k] - b[k]).abs().max().item() for k in a) < 1e-4


@pytest.mark.parametrize("n,args", [(2, ()), (2, ("--sp",)), (4, ("--sp",))])
def test_grad_norm_suite(n, args):
    run(n, "clip_suite.py", *args)


def test_grad_clip_cli_same_norm_across_layouts(tmp_path):
    """--grad-clip: the logged (pre-clip) global norm at step 0 is the same for
    one rank and for pp2 x tp2 (and training runs with clipping active)."""
    import json

    root = os.path.dirname(SUITES)
    train = os.path.join(os.path.dirname(root), "train.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    common = ["--layers", "4", "--heads", "4", "--embd", "64", "--block", "32", "--vocab", "256", "--batch", "4",
              "--micro", "2", "--steps", "3", "--grad-clip", "0.5", "--device", "cpu"]
    norms = {}
    for name, n, extra in [("single", 1, []), ("pp2tp2", 4, ["--pp", "2", "--tp", "2", "--sp"])]:
        sink = tmp_path / f"{name}.jsonl"
        assert launch(n, [train, *common, *extra, "--jsonl", str(sink)], timeout=300, env=env) == 0, name
        recs = [json.loads(ln) for ln in sink.read_text().splitlines()]
        norms[name] = recs[0]["grad_norm"]
    assert abs(norms["single"] - norms["pp2tp2"]) / norms["single"] < 1e-4, norms


def test_all_options_together(tmp_path):
    """dp2 x tp2 + SP with accumulation, block recompute, clipping, a cosine
    schedule, evaluation, background checkpoints, the step gate and heartbeats
    in one job."""
    import json

    from dstraining_b200.utils import checkpoint

    root = os.path.dirname(SUITES)
    train = os.path.join(os.path.dirname(root), "train.py")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    sink = tmp_path / "m.jsonl"
    argv = [train, "--dp", "2", "--tp", "2", "--sp", "--vp", "--recompute-blocks", "--grad-accum", "--micro", "2",
            "--batch", "4", "--layers", "2", "--heads", "4", "--embd", "64", "--block", "32", "--vocab", "256",
            "--steps", "6", "--grad-clip", "1.0", "--lr-schedule", "cosine", "--warmup-steps", "2",
            "--eval-every", "3", "--ckpt-dir", str(tmp_path / "ck"), "--ckpt-every", "2", "--ckpt-async",
            "--step-gate-timeout", "60", "--heartbeat-timeout", "120", "--jsonl", str(sink), "--device", "cpu"]
    assert launch(4, argv, timeout=400, env=env) == 0
    recs = [json.loads(ln) for ln in sink.read_text().splitlines()]
    assert sum("eval_loss" in r for r in recs) == 2 and all("grad_norm" in r for r in recs if "loss" in r)
    assert checkpoint.inspect(checkpoint.latest(str(tmp_path / "ck")))["ok"]
