"""Throughput benchmark: GPT-2 small (12L/768/12H, seq 1024, vocab 50304),
pure data parallelism dp=N, bf16 with fp32 master weights, micro-batch 16
per rank, 25 MB gradient buckets.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Protocol: W untimed warm-up steps, then K steps timed on the device with
CUDA events, bracketed by a barrier and a synchronize on both sides; the
step time is the max over ranks. Every step touches several GB (weights,
optimizer state, activations), far more than the 126 MB L2, so no explicit
L2 flush is needed. SM clocks and throttle reasons are sampled with
nvidia-smi during the timed region. A second timed loop runs the same steps
end to end through the public API (``Trainer.step``: pinned host batch ->
device copy -> step -> loss read back), which is the ``e2e`` figure.

``--impl reference`` runs the unmodified reference package installed under
``baseline/_ref`` through its own public API (its GPT, MasterWeightOptimizer,
GradReducer and SyntheticShard), timed identically. Rank 0 prints one JSON
line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
MODEL = dict(layers=12, heads=12, embd=768, block=1024, vocab=50304)
MICRO = 16
# Published reference numbers for GPT-2 124M (RTX 4090, docs/WRITEUP.md:311-312):
# 1 GPU 41.6k tok/s, dp=2 bucketed 75.4k tok/s. No B200 numbers are published.
PUBLISHED = {1: 41600.0, 2: 75400.0}
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """Samples SM clocks / throttle reasons of the visible GPUs with
    nvidia-smi every 200 ms while active."""

    def __init__(self):
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        q = "index,clocks.sm,clocks.max.sm,power.draw," + ",".join(f"clocks_event_reasons.{r}" for r in REASONS)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
        except FileNotFoundError:
            self.proc = None
            return

        def reader():
            for line in self.proc.stdout:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 4 + len(REASONS):
                    self.samples.append(parts)

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        active = set()
        for s in self.samples:
            for i, r in enumerate(REASONS):
                if s[4 + i].lower().startswith("active"):
                    active.add(r)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(active),
            "samples": len(self.samples),
        }


def setup_env():
    """Single-process runs get a one-rank rendezvous on 127.0.0.1 so both arms
    can use their own ``init_distributed`` unchanged."""
    if "RANK" not in os.environ:
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
    return int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])


def barrier():
    if dist.is_initialized():
        dist.barrier()


def max_over_ranks(x: float) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], device="cuda" if torch.cuda.is_available() else "cpu", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(fn, steps, sampler=None):
    """Device time per step (ms) of `steps` calls of fn(i), max over ranks."""
    barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        fn(i)
    end.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.stop()
    barrier()
    return max_over_ranks(start.elapsed_time(end) / steps)


def count_launches(step_fn, ours_marker):
    """Kernels launched by one step (profiled once, outside any timed region)."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn(0)
        torch.cuda.synchronize()
    ours = other = 0
    names = {}
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA:
            continue
        name = ev.name
        if any(m in name for m in ours_marker):
            ours += 1
        elif "Memcpy" in name or "Memset" in name:
            continue
        else:
            other += 1
            names[name[:60]] = names.get(name[:60], 0) + 1
    top_other = sorted(names.items(), key=lambda kv: -kv[1])[:8]
    return ours, other, top_other


# ---------------------------------------------------------------- our arm
def run_ours(a, rank, world):
    sys.path.insert(0, HERE)
    from dstraining_b200.trainer import Trainer, add_args

    targs = add_args(argparse.ArgumentParser()).parse_args([])
    targs.dp = world
    targs.bf16 = True
    targs.vp = True  # fused LM head + CE: the same loss as plain CE at tp=1
    targs.layers, targs.heads, targs.embd = MODEL["layers"], MODEL["heads"], MODEL["embd"]
    targs.block, targs.vocab = MODEL["block"], MODEL["vocab"]
    targs.batch = MICRO
    targs.seed = 1337
    tr = Trainer(targs)
    dev = tr.device
    batches = [tr.shard.get_batch(i, pin=True) for i in range(max(a.steps, a.warmup))]
    dev_batches = [(x.to(dev), y.to(dev)) for x, y in batches]
    for i in range(a.warmup):
        tr.step_device(*dev_batches[i % len(dev_batches)])
    torch.cuda.synchronize()
    sampler = ClockSampler() if rank == 0 else None
    losses = []

    def dev_step(i):
        losses.append(tr.step_device(*dev_batches[i]))

    ms = timed(dev_step, a.steps, sampler)
    final_loss = float(losses[-1].float().item())

    def e2e_step(i):
        tr.step(*batches[i])

    e2e_ms = timed(e2e_step, a.steps) if not a.no_e2e else float("nan")
    ours, other, top_other = (
        count_launches(lambda i: tr.step_device(*dev_batches[0]), ["dst::"]) if not a.no_count else (0, 0, [])
    )
    status = None
    from dstraining_b200.ops import native

    if native.available():
        status = int(native.lib().read_status(True))
    x0, y0 = batches[0]
    h2d = x0.numel() * x0.element_size() + y0.numel() * y0.element_size()
    return dict(
        ms=ms,
        e2e_ms=e2e_ms,
        loss=final_loss,
        launches=(ours, other, top_other),
        h2d=h2d,
        d2h=4,
        sampler=sampler,
        status=status,
        n_params=tr.n_params,
    )


# ---------------------------------------------------------------- reference arm
def run_reference(a, rank, world):
    ref_root = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "dst")):
        return {"unavailable": "reference not installed under baseline/_ref"}
    sys.path.insert(0, ref_root)
    for k in [k for k in sys.modules if k == "dst" or k.startswith("dst.")]:
        del sys.modules[k]
    from dst import parallel as rparallel  # the reference package
    from dst.data import SyntheticShard
    from dst.dp import GradReducer
    from dst.model import GPT, GPTConfig
    from dst.precision import MasterWeightOptimizer

    assert os.path.abspath(rparallel.__file__).startswith(os.path.abspath(ref_root))
    rparallel.init_distributed()
    tp, pp, dp = rparallel.make_topology(1, 1, world)
    dev = rparallel.default_device()
    cfg = GPTConfig(
        vocab_size=MODEL["vocab"],
        block_size=MODEL["block"],
        n_layer=MODEL["layers"],
        n_head=MODEL["heads"],
        n_embd=MODEL["embd"],
        dropout=0.0,
    )
    model = GPT(cfg, tp, seed=1337).to(dev).to(torch.bfloat16)
    opt = MasterWeightOptimizer(model.parameters(), lr=3e-4)
    reducer = GradReducer(model, dp) if dp.enabled else None
    shard = SyntheticShard(cfg.vocab_size, cfg.block_size, MICRO, seed=1337, dp=dp)
    batches = [tuple(t.pin_memory() for t in shard.get_batch(i)) for i in range(max(a.steps, a.warmup))]
    dev_batches = [(x.to(dev), y.to(dev)) for x, y in batches]

    def step_device(idx, tgt):
        opt.zero_grad(set_to_none=True)
        _, loss = model(idx, tgt)
        loss.backward()
        if reducer is not None:
            reducer.finish()
        model.finalize_grads()
        opt.step()
        return loss

    for i in range(a.warmup):
        step_device(*dev_batches[i % len(dev_batches)])
    torch.cuda.synchronize()
    sampler = ClockSampler() if rank == 0 else None
    losses = []
    ms = timed(lambda i: losses.append(step_device(*dev_batches[i])), a.steps, sampler)
    final_loss = float(losses[-1].float().item())

    def e2e_step(i):
        x, y = batches[i]
        loss = step_device(x.to(dev, non_blocking=True), y.to(dev, non_blocking=True))
        loss.float().item()

    e2e_ms = timed(e2e_step, a.steps) if not a.no_e2e else float("nan")
    x0, y0 = batches[0]
    return dict(
        ms=ms,
        e2e_ms=e2e_ms,
        loss=final_loss,
        launches=None,
        h2d=x0.numel() * x0.element_size() + y0.numel() * y0.element_size(),
        d2h=4,
        sampler=sampler,
        status=None,
        n_params=sum(p.numel() for p in model.parameters()),
    )


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-count", action="store_true", help="skip the profiled launch count (for ncu runs)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end loop (for ncu runs)")
    a = ap.parse_args()
    if a.warmup < 3:
        a.warmup = 3
    rank, world = setup_env()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but world size {world}")
    res = run_reference(a, rank, world) if a.impl == "reference" else run_ours(a, rank, world)
    if "unavailable" in res:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}), flush=True)
        return
    tokens = MICRO * MODEL["block"] * world
    value = tokens / (res["ms"] / 1000.0)
    e2e = tokens / (res["e2e_ms"] / 1000.0)
    pub = PUBLISHED.get(world)
    out = {
        "metric": "tokens/sec (whole box, device-timed, max over ranks)",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(res["ms"], 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(value / pub, 3) if pub else None,
        "dtype": "bf16",
        "data": "synthetic (uniform random token ids, seeded; random-init weights)",
        "config": {
            "model": "GPT-2 small 12L/768/12H, d_ff 3072, seq 1024, vocab 50304 (BASELINE config 2)",
            "global_batch": MICRO * world,
            "micro_batch_per_rank": MICRO,
            "seq_len": MODEL["block"],
            "parallelism": f"dp{world}",
            "optimizer": "Adam on fp32 masters, bf16 params (MasterWeightOptimizer)",
            "dp_buckets_mb": 25,
            "l2": "no flush: each step streams several GB of weights/optimizer state/activations (>> 126 MB L2)",
            "params": res["n_params"],
            "final_loss": round(res["loss"], 4),
        },
        "e2e": {
            "value": round(e2e, 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": res["h2d"],
            "d2h_bytes_per_step": res["d2h"],
            "ms_per_step": round(res["e2e_ms"], 3),
        },
    }
    if res["sampler"] is not None:
        out["clocks"] = res["sampler"].summary()
    if a.impl == "reference":
        out["impl"] = "reference"
        out["gpu_launches"] = None
    else:
        out["impl"] = "ours"
        ours, other, top_other = res["launches"]
        out["gpu_launches"] = ours * a.steps
        out["launches_per_step"] = {"ours": ours, "other": other, "top_other": top_other}
        out["device_status"] = res["status"]
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
