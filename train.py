"""Train a GPT with any composition of tp x pp x dp, interleaving, sequence
parallelism, selective recompute and bf16 + fp32 master weights.

    # CPU smoke test, all axes at once (8 gloo ranks):
    python -m dstraining_b200.utils.launch 8 train.py --dp 2 --pp 2 --tp 2 --chunks 2 \
        --sp --recompute --steps 20 --data synthetic
    # 8 B200s, GPT-2 124M data parallel, bf16 + fp32 masters:
    torchrun --nproc_per_node 8 train.py --dp 8 --bf16 --vp --gpt2 --batch 16

Same flags as the reference's ``train.py:29-58`` (plus ``--bucket-mb``,
checkpointing with retention and ``--save-on-signal`` (preemption), ``--profile-dir`` (a ``torch.profiler`` trace per rank), ``--bench`` (device-timed throughput over the steps after
``--bench-warmup``, max over ranks), ``--heartbeat-timeout`` and ``--jsonl``, whose records carry
the loss, tok/s, the device step time max over ranks, the peak memory and
the kernels' status word). Logs ``step N  loss X  T tok/s`` from the
last pipeline stage's tp0/dp0 rank; the loss is averaged over DP and the
throughput is over the steps since the previous log line, measured with the
device synchronised.
"""

import json
import sys
import time

import torch
import torch.distributed as dist

from dstraining_b200.ops import native
from dstraining_b200.parallel.health import StopRequest, maybe_inject_fault
from dstraining_b200.trainer import Trainer, parse_args
from dstraining_b200.utils import checkpoint
from dstraining_b200.utils.trace import StepProfiler


def main():
    args = parse_args()
    try:
        run(args)
    except Exception as e:  # tell the peers before dying, so they stop waiting
        if dist.is_initialized():
            from dstraining_b200.parallel.health import report_failure

            report_failure(f"{type(e).__name__}: {e}")
        raise


def bench_mark(cuda: bool):
    """A point in the device's timeline (CUDA event) or, on CPU, the host clock."""
    if cuda:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev
    return time.perf_counter()


def report_bench(args, tr, start, end, steps: int, sink) -> None:
    """``--bench``: mean step time over the timed window, max over all ranks,
    and the whole job's tokens/s (a collective: every rank calls it)."""
    if start is None or steps <= 0:
        ms = float("nan")
    elif isinstance(start, float):
        ms = (end - start) * 1e3 / steps
    else:
        end.synchronize()
        ms = start.elapsed_time(end) / steps
    (ms,) = tr.world_max([ms])
    if tr.is_logger:
        tps = tr.tokens_per_step / (ms / 1e3) if ms == ms else float("nan")
        print(f"bench  {steps} steps  {ms:.3f} ms/step (device, max over ranks)  {tps:,.0f} tok/s", flush=True)
        if sink:
            sink.write(json.dumps({"bench_steps": steps, "bench_ms_per_step": ms, "bench_tok_s": tps}) + "\n")
            sink.flush()


def prune(args) -> None:
    """Checkpoint retention (``--ckpt-keep``), by global rank 0 once a
    checkpoint is complete."""
    if args.ckpt_keep and (not dist.is_initialized() or dist.get_rank() == 0):
        checkpoint.prune(args.ckpt_dir, args.ckpt_keep)


def run(args):
    tr = Trainer(args)
    start_step = 0
    if args.resume and args.ckpt_dir:
        path = checkpoint.latest(args.ckpt_dir)
        if path:
            manifest = checkpoint.load(path, tr.model, tr.opt, tr.tp)
            start_step = int(manifest["step"])
            tr.step_index = start_step  # schedules and the step gate continue from here
            if tr.is_logger:
                print(f"resumed from {path} at step {start_step}", flush=True)
    if tr.is_logger:
        print(
            f"tp={args.tp} pp={args.pp} dp={args.dp} chunks={args.chunks} sp={args.sp} "
            f"recompute={args.recompute} bf16={args.bf16} vp={args.vp} device={tr.device.type} | "
            f"{tr.n_params:,} params this rank | batch {args.batch}/replica",
            flush=True,
        )
    sink = open(args.jsonl, "a") if (args.jsonl and tr.is_logger) else None
    cuda = tr.device.type == "cuda"
    events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) if cuda else None
    t_last, s_last = time.time(), start_step
    pending = None  # checkpoint being written in the background
    first_timed = start_step + args.bench_warmup
    window = None  # --bench: start/end marks around the timed steps
    stop = StopRequest() if (args.save_on_signal or args.time_limit_min) else None
    if stop and not args.ckpt_dir:
        raise SystemExit("--save-on-signal / --time-limit-min need --ckpt-dir")
    t_start = time.time()
    prof = None
    if args.profile_dir:
        p_start, p_count = (int(x) for x in args.profile_steps.split(":"))
        prof = StepProfiler(args.profile_dir, p_start, p_count, dist.get_rank() if dist.is_initialized() else 0,
                            cuda)
    for step in range(start_step, args.steps):
        maybe_inject_fault(step)
        if args.bench and step == first_timed:
            window = bench_mark(cuda)
        if prof:
            prof.before(step)
        idx, tgt = tr.shard.get_batch(step, pin=cuda)
        t_step = time.perf_counter()
        if events:
            events[0].record()
        loss = tr.step_device(idx.to(tr.device, non_blocking=True), tgt.to(tr.device, non_blocking=True))
        if events:
            events[1].record()
        if prof:
            prof.after(step)
        last = step == args.steps - 1
        logging = step % args.log_every == 0 or last
        record = None
        if args.jsonl and logging:
            # every rank: this step's device time (CPU: host time) and the
            # kernels' status word, reduced to the max over all ranks
            if events:
                events[1].synchronize()
                ms = events[0].elapsed_time(events[1])
            else:
                ms = (time.perf_counter() - t_step) * 1e3
            status = 0
            if cuda and native.available():
                status = int(native.lib().read_status(False))
            ms_max, status_max = tr.world_max([ms, status])
            record = {"step_ms_max": round(ms_max, 3), "status": int(status_max)}
            if tr.last_grad_norm is not None:
                record["grad_norm"] = tr.last_grad_norm  # before clipping
            if cuda:
                record["max_mem_gb"] = round(torch.cuda.max_memory_allocated(tr.device) / 2**30, 3)
        if tr.pp.is_last and logging:
            avg = tr.dp_mean_loss(loss)
            if tr.is_logger:
                value = avg.item()  # synchronises the device
                now = time.time()
                tps = tr.tokens_per_step * (step + 1 - s_last) / max(now - t_last, 1e-9)
                print(f"step {step:5d}  loss {value:.4f}  {tps:,.0f} tok/s", flush=True)
                if sink:
                    sink.write(json.dumps({"step": step, "loss": value, "tok_s": tps, **(record or {})}) + "\n")
                    sink.flush()
                t_last, s_last = now, step + 1
        if args.eval_every and ((step + 1) % args.eval_every == 0 or last):
            with tr.hold():
                ev = tr.eval_loss(args.eval_batches)  # every rank takes part
            if tr.is_logger:
                print(f"eval step {step:5d}  loss {ev:.4f}", flush=True)
                if sink:
                    sink.write(json.dumps({"step": step, "eval_loss": ev}) + "\n")
                    sink.flush()
        if stop is not None:
            stop.maybe_inject(step)
            if args.time_limit_min and time.time() - t_start > args.time_limit_min * 60:
                stop.flag = True
            if ((step + 1) % max(1, args.signal_check_every) == 0 or last) and stop.agreed(tr.device):
                with tr.hold():
                    if pending is not None:
                        pending.wait()
                    path = checkpoint.save(args.ckpt_dir, step + 1, tr.model, tr.opt, tr.tp, tr.pp, tr.dp,
                                           tr.config, args.seed)
                prune(args)
                if tr.is_logger:
                    print(f"stop requested (signal or time limit): saved {path} after step {step}; exiting",
                          flush=True)
                if prof:
                    prof.close()
                if sink:
                    sink.close()
                if dist.is_initialized():
                    dist.barrier()
                    dist.destroy_process_group()
                sys.exit(0)
        if args.ckpt_dir and args.ckpt_every and (step + 1) % args.ckpt_every == 0 and not last:
            with tr.hold():
                if pending is not None:
                    pending.wait()  # one background write at a time
                    prune(args)
                out = checkpoint.save(args.ckpt_dir, step + 1, tr.model, tr.opt, tr.tp, tr.pp, tr.dp, tr.config,
                                      args.seed, background=args.ckpt_async)
            pending = out if args.ckpt_async else None
            if pending is None:
                prune(args)
    if prof:
        prof.close()
    if args.bench:
        report_bench(args, tr, window, bench_mark(cuda) if window is not None else None, args.steps - first_timed,
                     sink)
    with tr.hold():
        if pending is not None:
            pending.wait()
        if args.ckpt_dir:
            checkpoint.save(args.ckpt_dir, args.steps, tr.model, tr.opt, tr.tp, tr.pp, tr.dp, tr.config, args.seed)
            prune(args)
    if sink:
        sink.close()
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    sys.exit(0)


if __name__ == "__main__":
    main()
