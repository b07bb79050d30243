"""Trainer / train.py plumbing on CPU (fp32 oracle path)."""

import argparse
import os

import pytest
import torch


@pytest.fixture()
def single_rank(monkeypatch, tmp_path):
    import torch.distributed as dist

    monkeypatch.setenv("DST_INIT_METHOD", f"file://{tmp_path}/store")
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    yield
    if dist.is_initialized():
        dist.destroy_process_group()


def test_trainer_loss_falls(single_rank):
    from dstraining_b200.trainer import Trainer, add_args

    a = add_args(argparse.ArgumentParser()).parse_args(["--device", "cpu", "--layers", "2", "--batch", "4", "--lr", "1e-3"])
    tr = Trainer(a)
    x, y = tr.shard.get_batch(0)
    losses = [tr.step(x, y) for _ in range(8)]
    assert losses[-1] < losses[0]
    assert tr.tokens_per_step == 4 * 64


def test_weight_decay_is_adamw(single_rank):
    """--weight-decay gives decoupled (AdamW) decay: three trainer steps equal
    torch.optim.AdamW (same fused CPU kernel, so bitwise) on a copy of the
    model fed the same batches."""
    import copy

    from dstraining_b200.trainer import Trainer, add_args

    a = add_args(argparse.ArgumentParser()).parse_args(
        ["--device", "cpu", "--layers", "1", "--batch", "2", "--lr", "1e-2", "--weight-decay", "0.5"])
    tr = Trainer(a)
    ref = copy.deepcopy(tr.model)
    opt = torch.optim.AdamW(ref.parameters(), lr=1e-2, weight_decay=0.5, fused=True)  # the trainer's CPU kernel
    for s in range(3):
        x, y = tr.shard.get_batch(s)
        tr.step(x, y)
        opt.zero_grad(set_to_none=True)
        ref(x, y)[1].backward()
        opt.step()
    for (n, p), q in zip(tr.model.named_parameters(), ref.parameters()):
        assert torch.equal(p, q), n


def test_master_weights_take_torch_path_for_weight_decay():
    """Adam options the native kernel lacks run the PyTorch update of the same
    step (the reference passes every Adam keyword to torch.optim.Adam)."""
    from dstraining_b200.optim.precision import MasterWeightOptimizer

    torch.manual_seed(0)
    w = torch.nn.Parameter(torch.randn(64, 32).to(torch.bfloat16))
    opt = MasterWeightOptimizer([w], lr=1e-2, weight_decay=0.1)
    master = w.detach().float().clone().requires_grad_(True)
    ref = torch.optim.Adam([master], lr=1e-2, weight_decay=0.1)
    for _ in range(3):
        g = torch.randn(64, 32).to(torch.bfloat16)
        w.grad = g
        master.grad = g.float()
        opt.step()
        ref.step()
    torch.testing.assert_close(opt.master_params[0], master.detach(), atol=0, rtol=0)
    assert torch.equal(w.detach(), master.detach().to(torch.bfloat16))


def test_train_bench_record(tmp_path):
    """``train.py --bench``: one record with the device (here: host) step time
    over the steps after the warm-up, max over ranks, and the job's tok/s."""
    import json

    from dstraining_b200.utils.launch import launch

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sink = tmp_path / "m.jsonl"
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    argv = [os.path.join(root, "train.py"), "--dp", "2", "--layers", "1", "--heads", "2", "--embd", "32", "--block",
            "32", "--vocab", "128", "--batch", "2", "--steps", "6", "--device", "cpu", "--bench", "--bench-warmup",
            "2", "--log-every", "10", "--jsonl", str(sink)]
    assert launch(2, argv, timeout=300, env=env) == 0
    rec = [json.loads(line) for line in sink.read_text().splitlines() if "bench_steps" in line]
    assert len(rec) == 1 and rec[0]["bench_steps"] == 4 and rec[0]["bench_ms_per_step"] > 0
    assert abs(rec[0]["bench_tok_s"] - 2 * 32 * 2 / (rec[0]["bench_ms_per_step"] / 1e3)) < 1e-3 * rec[0]["bench_tok_s"]


def test_train_profile_window(tmp_path):
    """``train.py --profile-dir``: one Chrome trace per rank, holding the
    trainer's phase ranges and the blocks of the profiled steps."""
    import json

    from dstraining_b200.utils.launch import launch

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    argv = [os.path.join(root, "train.py"), "--dp", "2", "--layers", "2", "--heads", "2", "--embd", "32", "--block",
            "32", "--vocab", "128", "--batch", "2", "--steps", "5", "--device", "cpu", "--profile-dir",
            str(tmp_path / "prof"), "--profile-steps", "2:2", "--log-every", "10"]
    assert launch(2, argv, timeout=300, env=env) == 0
    for r in range(2):
        trace = json.loads((tmp_path / "prof" / f"trace_rank{r}.json").read_text())
        names = [e.get("name") for e in trace["traceEvents"]]
        assert names.count("forward_backward") == 2 and names.count("optimizer") == 2
        assert names.count("block1") == 2


def test_fused_dp_adam_weight_decay_is_adamw():
    """FusedDPAdam's decoupled weight decay (host path; the native kernels
    apply the same factor) equals torch.optim.AdamW."""
    import copy

    from dstraining_b200.models.gpt import GPT, GPTConfig
    from dstraining_b200.optim.fused_dp import FusedDPAdam
    from dstraining_b200.parallel.topology import SINGLE

    cfg = GPTConfig(vocab_size=128, block_size=16, n_layer=1, n_head=2, n_embd=32)
    m = GPT(cfg, SINGLE, seed=2)
    ref = copy.deepcopy(m)
    opt = FusedDPAdam(m, SINGLE, lr=1e-2, weight_decay=0.3, bucket_bytes=1 << 12)
    ref_opt = torch.optim.AdamW(ref.parameters(), lr=1e-2, weight_decay=0.3)
    g = torch.Generator().manual_seed(0)
    for _ in range(3):
        x, y = torch.randint(0, 128, (2, 16), generator=g), torch.randint(0, 128, (2, 16), generator=g)
        opt.zero_grad()
        m(x, y)[1].backward()
        opt.step()
        ref_opt.zero_grad()
        ref(x, y)[1].backward()
        ref_opt.step()
    for (n, p), q in zip(m.named_parameters(), ref.parameters()):
        assert (p - q).abs().max().item() < 1e-5, n


def test_device_busy_time_counts_overlaps_once():
    from dstraining_b200.utils.trace import busy_time

    # two streams overlapping on [2, 3), a gap [5, 6), a span nested in another
    assert busy_time([(0.0, 3.0), (2.0, 5.0), (6.0, 10.0), (7.0, 8.0)]) == 9.0
    assert busy_time([(1.0, 2.0)]) == 1.0
