"""Training-step API shared by ``train.py`` and ``bench.py``.

``Trainer(args)`` builds the process grid, the model (``GPT`` / ``GPTStage``
/ ``GPTChunks``), the schedule, the optimizer and the gradient reducer from a
``train.py``-style argument namespace, mirroring the reference's
``train.py:61-110``. One optimisation step is

    zero_grad -> forward/backward (or pipeline train_step) -> DP reduce ->
    finalize_grads (SP) -> optimizer step

``step_device(idx, tgt)`` runs it on tensors already on the device and returns
the loss tensor (``None`` off the last stage); ``step(idx, tgt)`` is the end-to-
end call a user makes: it copies a (pinned) host batch to the device, runs the
step and reads the loss back to the host.
"""

from __future__ import annotations

import argparse
import os
from typing import Optional

import torch
import torch.distributed as dist

from .models.gpt import GPT, GPTChunks, GPTConfig, GPTStage
from .optim.clip import clip_grad_norm
from .optim.fused_dp import FusedDPAdam
from .optim.precision import MasterWeightOptimizer
from .optim.schedule import lr_at, set_lr
from .parallel import topology
from .parallel.dp import GradReducer, allreduce_gradients
from .parallel.pipeline import Pipeline1F1B, PipelineInterleaved
from .utils.data import SyntheticShard, TokenShard
from .utils.trace import nvtx_range


def add_args(p: argparse.ArgumentParser) -> argparse.ArgumentParser:
    """The reference's ``train.py`` flags (``train.py:29-58``) plus bucket size
    and checkpointing."""
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--chunks", type=int, default=1, help="model chunks per rank (v > 1: interleaved)")
    p.add_argument("--sp", action="store_true", help="sequence parallelism")
    p.add_argument("--recompute", action="store_true", help="selective attention recompute")
    p.add_argument("--recompute-blocks", action="store_true",
                   help="full activation recompute: each block keeps only its input")
    p.add_argument("--bf16", action="store_true", help="bf16 params + fp32 master weights")
    p.add_argument("--vp", action="store_true", help="vocab-parallel (fused) cross-entropy")
    p.add_argument("--naive-dp", action="store_true", help="per-parameter blocking all-reduce")
    p.add_argument("--gpt2", action="store_true", help="GPT-2 124M shape")
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--embd", type=int, default=128)
    p.add_argument("--block", type=int, default=64)
    p.add_argument("--vocab", type=int, default=512)
    p.add_argument("--data", default="synthetic", help="'synthetic' or a uint16 token file")
    p.add_argument("--batch", type=int, default=8, help="batch per DP replica")
    p.add_argument("--micro", type=int, default=1, help="micro batch size (pipelines; with --grad-accum also pp=1)")
    p.add_argument("--grad-accum", action="store_true",
                   help="without pipelining: split each batch into --micro-sized micro-batches and accumulate")
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--lr", type=float, default=3e-4)
    p.add_argument("--lr-schedule", choices=["constant", "cosine"], default="constant")
    p.add_argument("--warmup-steps", type=int, default=0, help="linear learning-rate warm-up")
    p.add_argument("--min-lr", type=float, default=0.0, help="final rate of the cosine schedule")
    p.add_argument("--weight-decay", type=float, default=0.0,
                   help="decoupled (AdamW) weight decay (0: plain Adam, as the reference)")
    p.add_argument("--grad-clip", type=float, default=0.0,
                   help="clip the global gradient norm to this value (0: off; not with the fused DP optimizer)")
    p.add_argument("--seed", type=int, default=1337)
    p.add_argument("--log-every", type=int, default=1)
    p.add_argument("--device", default=None, help="cuda|cpu (default: cuda if available)")
    p.add_argument("--bucket-mb", type=float, default=25.0, help="DP gradient bucket size")
    p.add_argument("--ckpt-dir", default=None, help="directory for sharded checkpoints")
    p.add_argument("--ckpt-every", type=int, default=0, help="save every N steps (0: only at the end if --ckpt-dir)")
    p.add_argument("--resume", action="store_true", help="resume from the latest checkpoint in --ckpt-dir")
    p.add_argument("--ckpt-keep", type=int, default=0,
                   help="keep only the newest N complete checkpoints (0: keep all)")
    p.add_argument("--save-on-signal", action="store_true",
                   help="on SIGTERM / SIGUSR1 to any rank: checkpoint at the next agreed step and exit 0")
    p.add_argument("--time-limit-min", type=float, default=0.0,
                   help="checkpoint and exit 0 once this much wall time has passed (0: off; needs --ckpt-dir)")
    p.add_argument("--signal-check-every", type=int, default=10,
                   help="steps between the (collective) checks for a pending signal or time limit")
    p.add_argument("--ckpt-async", action="store_true",
                   help="write periodic checkpoints from a background thread (training continues)")
    p.add_argument("--jsonl", default=None, help="append per-step metrics (JSON lines) to this file")
    p.add_argument("--profile-dir", default=None,
                   help="write a torch.profiler Chrome trace per rank for the --profile-steps window")
    p.add_argument("--profile-steps", default="5:3", help="START:COUNT of the profiled window")
    p.add_argument("--bench", action="store_true",
                   help="report device-timed throughput over the steps after --bench-warmup (max over ranks)")
    p.add_argument("--bench-warmup", type=int, default=3, help="untimed steps before the --bench window")
    p.add_argument("--eval-data", default=None,
                   help="held-out uint16 token file ('synthetic': a separately seeded random stream)")
    p.add_argument("--eval-every", type=int, default=0, help="evaluate every N steps (0: off)")
    p.add_argument("--eval-batches", type=int, default=4, help="batches per evaluation")
    p.add_argument("--heartbeat-timeout", type=float, default=0.0,
                   help="abort when a peer makes no progress for this many seconds (0: off)")
    p.add_argument("--step-gate-timeout", type=float, default=0.0,
                   help="before each step, wait at most this long for every rank to reach it; "
                        "raise PeerFailure otherwise (0: off)")
    return p


def parse_args(argv=None) -> argparse.Namespace:
    """``train.py`` arguments; ``--config FILE.yaml`` supplies defaults for any
    flag (keys are flag names, with ``-`` or ``_``), and flags given on the
    command line take precedence."""
    pre = argparse.ArgumentParser(add_help=False)
    pre.add_argument("--config", default=None)
    known, _ = pre.parse_known_args(argv)
    p = add_args(argparse.ArgumentParser())
    p.add_argument("--config", default=None, help="YAML file of flag defaults (command line wins)")
    if known.config:
        import yaml

        with open(known.config) as f:
            conf = yaml.safe_load(f) or {}
        dests = {a.dest for a in p._actions}
        defaults = {}
        for k, v in conf.items():
            d = str(k).replace("-", "_")
            if d not in dests:
                raise ValueError(f"{known.config}: unknown flag {k!r}")
            defaults[d] = v
        p.set_defaults(**defaults)
    return p.parse_args(argv)


class Trainer:
    """Builds grid, model, schedule, optimizer and reducer from ``train.py``-style
    arguments (module docstring) and runs optimisation steps."""

    def __init__(self, args: argparse.Namespace):
        topology.init_distributed()
        self.args = args
        self.tp, self.pp, self.dp = topology.make_topology(args.tp, args.pp, args.dp)
        self.device = torch.device(args.device) if args.device else topology.default_device()
        if args.gpt2:
            args.layers, args.heads, args.embd, args.block, args.vocab = 12, 12, 768, 1024, 50257
        self.config = GPTConfig(
            vocab_size=args.vocab,
            block_size=args.block,
            n_layer=args.layers,
            n_head=args.heads,
            n_embd=args.embd,
            sequence_parallel=args.sp,
            recompute_attention=args.recompute,
            vocab_parallel_loss=args.vp,
            recompute_blocks=getattr(args, "recompute_blocks", False),
        )
        cfg = self.config
        if args.chunks > 1:
            model = GPTChunks(cfg, self.tp, self.pp, v=args.chunks, seed=args.seed)
        elif args.pp > 1:
            model = GPTStage(cfg, self.tp, self.pp, seed=args.seed)
        else:
            model = GPT(cfg, self.tp, seed=args.seed)
        model = model.to(self.device)
        if args.bf16:
            model = model.to(torch.bfloat16)
        self.model = model
        if args.chunks > 1:
            self.pipe = PipelineInterleaved(model, self.pp, micro_batch_size=args.micro, seq_len=cfg.block_size)
        elif args.pp > 1:
            self.pipe = Pipeline1F1B(model, self.pp, micro_batch_size=args.micro, seq_len=cfg.block_size)
        else:
            self.pipe = None
        cuda = self.device.type == "cuda"
        if cuda:
            # whether each group's ranks can address each other's GPU memory (one
            # host): collectives, made here by every rank in the same order, so
            # the answer is cached before any forward pass asks for it
            topology.peer_reachable(self.tp)
            topology.peer_reachable(self.dp)
        self.fused_dp = args.bf16 and not args.naive_dp and cuda and os.environ.get("DST_FUSED_DP", "1") != "0"
        if self.fused_dp:
            # DP reduction + fp32-master Adam + parameter all-gather per bucket,
            # launched on a side stream as backward finishes each bucket, with
            # the optimizer state sharded over DP: one NVLink kernel when every
            # DP rank is on this host, the group's collectives (NCCL reduce-
            # scatter / all-gather around the native Adam) otherwise. With a
            # single replica the kernel is the bucketed Adam update.
            self.opt = FusedDPAdam(
                model, self.dp, lr=args.lr, bucket_bytes=int(args.bucket_mb * 1024 * 1024), overlap=self.pipe is None,
                weight_decay=getattr(args, "weight_decay", 0.0),
            )
        else:
            wd = getattr(args, "weight_decay", 0.0)
            decay = dict(weight_decay=wd, decoupled_weight_decay=True) if wd else {}
            if args.bf16:
                self.opt = MasterWeightOptimizer(model.parameters(), lr=args.lr, **decay)
            else:
                # fused Adam (one vectorised pass per tensor; on CPU about 3x faster than
                # the multi-tensor loop, the default there); same update as torch.optim.Adam
                self.opt = torch.optim.Adam(model.parameters(), lr=args.lr, fused=True, **decay)
        if getattr(args, "grad_clip", 0.0) and self.fused_dp:
            raise ValueError("--grad-clip needs the unfused optimizer path (the fused DP optimizer updates "
                             "inside backward); set DST_FUSED_DP=0 or --naive-dp")
        self.last_grad_norm = None
        self.reducer = None
        if self.dp.enabled and not args.naive_dp and not self.fused_dp:
            self.reducer = GradReducer(
                model, self.dp, bucket_bytes=int(args.bucket_mb * 1024 * 1024), overlap=self.pipe is None
            )
        if args.data == "synthetic":
            self.shard = SyntheticShard(cfg.vocab_size, cfg.block_size, args.batch, seed=args.seed, dp=self.dp)
        else:
            self.shard = TokenShard(args.data, cfg.block_size, args.batch, seed=args.seed, dp=self.dp)
        self.accum = 1
        if getattr(args, "grad_accum", False) and self.pipe is None and args.micro < args.batch:
            if args.batch % args.micro:
                raise ValueError(f"batch {args.batch} not divisible by micro batch {args.micro}")
            self.accum = args.batch // args.micro
        self.tokens_per_step = args.batch * cfg.block_size * args.dp
        self.is_logger = self.pp.is_last and self.tp.rank == 0 and self.dp.rank == 0
        self.step_index = 0
        self.heartbeat = self.watchdog = self.gate = None
        if getattr(args, "step_gate_timeout", 0.0) and dist.is_initialized() and dist.get_world_size() > 1:
            from .parallel.health import StepGate

            self.gate = StepGate(timeout=args.step_gate_timeout)
        if getattr(args, "heartbeat_timeout", 0.0) and dist.is_initialized() and dist.get_world_size() > 1:
            from .parallel.health import start_monitoring

            hb_timeout = args.heartbeat_timeout
            self.heartbeat, self.watchdog = start_monitoring(interval=min(1.0, hb_timeout / 4), timeout=hb_timeout)

    def hold(self):
        """Context for a long phase between steps (checkpoint, evaluation): the
        heartbeat keeps publishing meanwhile (no-op without ``--heartbeat-timeout``)."""
        import contextlib

        return self.heartbeat.hold() if self.heartbeat is not None else contextlib.nullcontext()

    @property
    def n_params(self) -> int:
        return sum(p.numel() for p in self.model.parameters())

    def step_device(self, idx: torch.Tensor, tgt: torch.Tensor) -> Optional[torch.Tensor]:
        """One optimisation step on device tensors ``idx`` / ``tgt`` of this replica's
        batch; returns the (batch-mean) loss tensor on the last stage, else ``None``."""
        if self.gate is not None:
            self.gate.enter(self.step_index)  # host side, before this step launches anything
        a = self.args
        if getattr(a, "lr_schedule", "constant") != "constant" or getattr(a, "warmup_steps", 0):
            # before backward: the fused optimizer launches buckets during it
            set_lr(self.opt, lr_at(self.step_index, a.lr, a.steps, a.warmup_steps, a.lr_schedule, a.min_lr))
        self.opt.zero_grad(set_to_none=True)
        with nvtx_range("forward_backward"):
            if self.pipe is not None:
                loss = self.pipe.train_step(idx, tgt)
                if self.reducer is not None:
                    self.reducer.reduce()
            elif self.accum > 1:
                loss = self._accumulate(idx, tgt)
            else:
                _, loss = self.model(idx, tgt)
                loss.backward()
        with nvtx_range("dp_reduce"):
            if self.reducer is not None:
                self.reducer.finish()
            elif self.dp.enabled and not self.fused_dp:
                allreduce_gradients(self.model, self.dp)
        with nvtx_range("finalize_grads"):
            self.model.finalize_grads()
        if getattr(a, "grad_clip", 0.0):
            self.last_grad_norm = clip_grad_norm(self.model, a.grad_clip, self.tp, self.dp)
        with nvtx_range("optimizer"):
            self.opt.step()
        self.step_index += 1
        if self.heartbeat is not None:
            self.heartbeat.tick()
        return loss

    def _accumulate(self, idx: torch.Tensor, tgt: torch.Tensor) -> torch.Tensor:
        """Forward/backward of ``accum`` micro-batches, gradients summed in
        ``param.grad`` (each loss scaled by 1/accum). The DP reducer's and the
        fused optimizer's hooks stay quiet until the last micro-batch, whose
        backward then reduces the accumulated gradients bucket by bucket."""
        hooked = [o for o in (self.reducer, self.opt) if hasattr(o, "defer")]
        xs, ys = idx.split(self.args.micro), tgt.split(self.args.micro)
        m = len(xs)
        total = None
        for i, (x, y) in enumerate(zip(xs, ys)):
            for o in hooked:
                o.defer = i < m - 1
            try:
                _, loss = self.model(x, y)
                (loss / m).backward()
            finally:
                for o in hooked:
                    o.defer = False
            part = loss.detach() / m
            total = part if total is None else total + part
        return total

    def step(self, idx: torch.Tensor, tgt: torch.Tensor) -> Optional[float]:
        """End-to-end step from host tensors; returns the local loss (host
        float) on the last pipeline stage, None elsewhere."""
        idx = idx.to(self.device, non_blocking=True)
        tgt = tgt.to(self.device, non_blocking=True)
        loss = self.step_device(idx, tgt)
        return None if loss is None else float(loss.detach().float().item())

    def world_max(self, values) -> list:
        """Element-wise max of a list of floats over every rank (a collective:
        all ranks must call it together)."""
        t = torch.tensor([float(v) for v in values], dtype=torch.float64,
                         device=self.device if self.device.type == "cuda" else "cpu")
        if dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def eval_loss(self, batches: int) -> Optional[float]:
        """Mean loss over ``batches`` held-out batches, forward only (pipelines
        run their forward-only schedule), averaged over DP. A collective over
        the whole job; returns the value on the last pipeline stage and
        ``None`` elsewhere."""
        a = self.args
        if getattr(self, "_eval_shard", None) is None:
            cfg, seed = self.config, a.seed + 7919  # a stream disjoint from the training batches
            if a.eval_data in (None, "synthetic"):
                self._eval_shard = SyntheticShard(cfg.vocab_size, cfg.block_size, a.batch, seed=seed, dp=self.dp)
            else:
                self._eval_shard = TokenShard(a.eval_data, cfg.block_size, a.batch, seed=seed, dp=self.dp)
        was_training = self.model.training
        self.model.eval()
        total = None
        try:
            for i in range(batches):
                x, y = self._eval_shard.get_batch(i)
                x, y = x.to(self.device), y.to(self.device)
                with torch.no_grad():
                    loss = self.pipe.eval_step(x, y) if self.pipe is not None else self.model(x, y)[1]
                if loss is not None:
                    part = loss.detach().float() / batches
                    total = part if total is None else total + part
        finally:
            self.model.train(was_training)
        if not self.pp.is_last:
            return None
        return float(self.dp_mean_loss(total).item())

    def dp_mean_loss(self, loss: torch.Tensor) -> torch.Tensor:
        """The loss averaged over the DP group (a collective; last-stage ranks)."""
        avg = loss.detach().float().clone()
        if self.dp.enabled:
            dist.all_reduce(avg, group=self.dp.group)
            avg /= self.dp.world
        return avg
