"""Data-parallel gradient reduction fused with the fp32-master Adam update.

``FusedDPAdam(model, dp, lr=..., betas=..., eps=...)`` replaces the pair
``GradReducer`` + ``MasterWeightOptimizer`` for bf16 models on CUDA. Parameters
are packed into ~25 MiB buckets in reverse registration order (roughly the
order backward finishes them). Each bucket owns two peer buffers
(:class:`dstraining_b200.parallel.symm.PeerBuffer`), one for its gradients and
one for its parameters; every parameter's ``.data`` becomes a view of the
parameter buffer. As backward finishes a bucket (post-accumulate-grad hooks
copy the gradients into its gradient buffer), the bucket's fused kernel is
launched on a side stream:

  each rank sums its 1/N slice of the bucket from all ranks' gradient buffers
  over NVLink (fixed rank order), scales by 1/N, applies Adam to its fp32
  master / moment slices, and stores the bf16 result into every rank's
  parameter buffer - reduce-scatter, optimizer and all-gather in one launch.

Adam state is therefore sharded (ZeRO-1: 1/N of the masters and moments per
rank) and the optimizer work per GPU shrinks with N. ``step()`` launches the
buckets that are still pending (all of them for pipeline schedules, which call
it after ``train_step``; the bucket of sequence-parallel partial-gradient
parameters always waits for ``finalize_grads``) and makes the compute stream
wait for the side stream. Buckets launch strictly in bucket order so every
rank issues the same kernel sequence.

Transports (``transport=``, chosen automatically by default):

* ``"peer"`` (CUDA, every DP rank on this host, at most 8): the fused NVLink
  kernel above;
* ``"collectives"`` (CUDA otherwise, e.g. DP groups spanning machines): the
  same buckets, hooks and ZeRO-1 sharding with the group's own collectives -
  an averaging reduce-scatter of the bucket (NCCL), the native multi-tensor
  Adam on the owned slice, an in-place all-gather of the bf16 parameters -
  issued on the side stream, so they still overlap the rest of backward (on
  gloo the same steps with PyTorch ops, for tests);
* ``"host"`` (no CUDA, gloo): all-reduce, Adam on the owned slice by PyTorch
  ops, all-gather - the CPU correctness path.

The update matches ``torch.optim.Adam`` (``torch.optim.AdamW`` with
``weight_decay``).
"""

from __future__ import annotations

from typing import List, Optional

import contextlib

import torch
import torch.distributed as dist

from ..ops import native
from ..parallel.comm import reduce_scatter_dim
from ..parallel.dp import build_buckets
from ..parallel.topology import DPContext, peer_reachable

_ALIGN = 8  # elements per rank slice are a multiple of this (16-byte vectors)


class _Bucket:
    def __init__(self, params, dp: DPContext, device, dtype, late: bool, use_peer: bool):
        self.params = params
        self.late = late
        self.offsets, off = [], 0
        for p in params:
            self.offsets.append(off)
            off += p.numel()
        self.numel = off
        n = dp.world
        self.slice = -(-off // (n * _ALIGN)) * _ALIGN
        self.padded = self.slice * n
        esize = torch.tensor([], dtype=dtype).element_size()
        if use_peer:
            from ..parallel.symm import PeerBuffer

            self.gbuf = PeerBuffer(self.padded * esize, dp, device)
            self.pbuf = PeerBuffer(self.padded * esize, dp, device)
            self.grad = self.gbuf.view(dtype)
            self.param = self.pbuf.view(dtype)
        else:
            self.gbuf = self.pbuf = None
            self.grad = torch.zeros(self.padded, dtype=dtype, device=device)
            self.param = torch.zeros(self.padded, dtype=dtype, device=device)
        with torch.no_grad():
            for p, o in zip(params, self.offsets):
                self.param[o : o + p.numel()].copy_(p.data.reshape(-1))
                p.data = self.param[o : o + p.numel()].view_as(p)
        lo = dp.rank * self.slice
        self.master = self.param[lo : lo + self.slice].float().clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.gshard = None if use_peer else torch.zeros(self.slice, dtype=dtype, device=device)
        self.filled = set()
        self.launched = False

    def slot(self, i):
        p = self.params[i]
        return self.grad[self.offsets[i] : self.offsets[i] + p.numel()].view_as(p)

    def stage(self, i) -> None:
        g = self.params[i].grad
        dst = self.slot(i)
        if g is None:
            dst.zero_()
        elif g.data_ptr() != dst.data_ptr():
            dst.copy_(g)

    def stage_all(self) -> None:
        """Copy every parameter's gradient into the bucket's gradient buffer
        with one multi-tensor copy (a handful of kernels instead of one copy
        per parameter)."""
        dsts, srcs = [], []
        for i, p in enumerate(self.params):
            g = p.grad
            dst = self.slot(i)
            if g is None:
                dst.zero_()
            elif g.data_ptr() != dst.data_ptr():
                dsts.append(dst)
                srcs.append(g)
        if dsts:
            torch._foreach_copy_(dsts, srcs)


class FusedDPAdam:
    """DP gradient averaging fused with fp32-master Adam (module docstring):
    ZeRO-1 sharded optimizer state, one NVLink kernel per bucket launched from
    backward hooks on CUDA, PyTorch collectives on gloo."""

    def __init__(
        self,
        model: torch.nn.Module,
        dp: DPContext,
        lr: float = 3e-4,
        betas=(0.9, 0.999),
        eps: float = 1e-8,
        bucket_bytes: int = 25 * 1024 * 1024,
        overlap: bool = True,
        transport: str = "auto",
        weight_decay: float = 0.0,
    ):
        self.dp = dp
        self.lr, self.betas, self.eps = lr, tuple(betas), eps
        self.weight_decay = float(weight_decay)  # decoupled (AdamW): master *= 1 - lr * weight_decay
        self.model_params = [p for p in model.parameters() if p.requires_grad]
        p0 = self.model_params[0]
        self.device, self.dtype = p0.device, p0.dtype
        self.native = p0.is_cuda and native.enabled()
        if self.native and self.dtype != torch.bfloat16:
            raise ValueError("DP Adam on CUDA needs bf16 parameters")
        if transport == "auto":
            if not self.native:
                transport = "host"
            else:
                # collective on the DP group the first time: every rank decides alike
                transport = "peer" if dp.world <= 8 and peer_reachable(dp) else "collectives"
        fits = {"peer": self.native, "collectives": True, "host": not self.native}
        if not fits.get(transport, False):
            raise ValueError(f"transport {transport!r} does not fit parameters on {p0.device}")
        if transport == "peer" and (dp.world > 8 or not peer_reachable(dp)):
            raise ValueError("the peer transport needs at most 8 DP ranks on this host, each with a GPU the "
                             "others can address (CUDA IPC)")
        self.transport = transport
        order = self.model_params[::-1]
        late = [p for p in order if getattr(p, "sequence_parallel_replicated", False)]
        early = [p for p in order if not getattr(p, "sequence_parallel_replicated", False)]
        groups = [(g, False) for g in build_buckets(early, bucket_bytes)] + ([(late, True)] if late else [])
        self.buckets: List[_Bucket] = [
            _Bucket(g, dp, self.device, self.dtype, is_late, transport == "peer") for g, is_late in groups
        ]
        self._where = {}
        for b in self.buckets:
            for i, p in enumerate(b.params):
                self._where[id(p)] = (b, i)
        self._next = 0  # next bucket to launch (buckets launch in order)
        self._step = 0
        self._stepped = False
        self.overlap = overlap
        self.defer = False  # set while accumulating gradients over micro-batches
        self.epoch = 0
        if transport == "peer":
            from ..parallel.symm import PeerBuffer

            self.flags = PeerBuffer(64 * 4, dp, self.device)
            self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        if self.native:
            self.side = torch.cuda.Stream(device=self.device)
        self.record_timings = False  # per-bucket CUDA events on the side stream (see timings())
        self._events = []
        self._tail = None
        if overlap:
            for p in order:
                p.register_post_accumulate_grad_hook(self._hook)

    # -- bookkeeping ------------------------------------------------------
    def zero_grad(self, set_to_none: bool = True) -> None:
        """Clear (or zero) the parameters' gradients."""
        for p in self.model_params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def _hook(self, p) -> None:
        if self.defer:
            return  # gradient accumulation: only the last micro-batch's backward launches buckets
        b, i = self._where[id(p)]
        if b.late:
            return  # staged in step(), after finalize_grads
        if not self.native:
            b.stage(i)
        b.filled.add(i)  # on CUDA the bucket is staged in one multi-tensor copy at launch
        self._launch_ready()

    def _launch_ready(self) -> None:
        while self._next < len(self.buckets):
            b = self.buckets[self._next]
            if b.late or len(b.filled) < len(b.params):
                return
            self._launch(b)
            self._next += 1

    def _launch(self, b: _Bucket) -> None:
        if not self._stepped:
            self._step += 1
            self._stepped = True
        b.launched = True
        if self.native:
            b.stage_all()
        timed = self.record_timings and self.native
        if timed:
            ev_stage = torch.cuda.Event(enable_timing=True)
            ev_stage.record(torch.cuda.current_stream(self.device))
        if self.transport == "peer":
            self._launch_native(b)
        elif self.transport == "collectives":
            self._launch_sharded(b)
        else:
            self._launch_emulated(b)
        if timed:
            ev_done = torch.cuda.Event(enable_timing=True)
            ev_done.record(self.side)
            self._events.append((self.buckets.index(b), b.numel, ev_stage, ev_done))

    def _launch_native(self, b: _Bucket) -> None:
        self.epoch += 1
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.side.wait_event(ev)
        with torch.cuda.stream(self.side):
            native.lib().fused_dp_adam(
                b.gbuf.ptrs, b.pbuf.ptrs, self.flags.ptrs, b.master, b.exp_avg, b.exp_avg_sq, self.done,
                b.slice, b.numel, self.dp.rank, self.epoch, self.lr, self.betas[0], self.betas[1], self.eps,
                float(self._step), weight_decay=self.weight_decay,
            )

    def _launch_sharded(self, b: _Bucket) -> None:
        """ZeRO-1 with the group's collectives (``collectives`` transport), ordered on the
        side stream after the compute stream's work so far: averaging
        reduce-scatter of the bucket into this rank's slice, Adam on the slice
        (native multi-tensor kernel on CUDA), in-place all-gather of the bf16
        parameters."""
        lo = self.dp.rank * b.slice
        valid = max(0, min(b.slice, b.numel - lo))
        cuda = self.native
        if cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.side.wait_event(ev)
        with torch.cuda.stream(self.side) if cuda else contextlib.nullcontext():
            if not self.dp.enabled:
                b.gshard.copy_(b.grad)
            elif cuda:
                dist.reduce_scatter_tensor(b.gshard, b.grad, op=dist.ReduceOp.AVG, group=self.dp.group)
            else:
                b.gshard.copy_(reduce_scatter_dim(b.grad, self.dp, 0) / self.dp.world)
            if valid:
                p_slice = b.param[lo : lo + valid]
                if cuda:
                    native.lib().adam_master_step(
                        [p_slice], [b.gshard[:valid]], [b.master[:valid]], [b.exp_avg[:valid]],
                        [b.exp_avg_sq[:valid]], self.lr, self.betas[0], self.betas[1], self.eps, float(self._step),
                        weight_decay=self.weight_decay,
                    )
                else:
                    self._adam(b, b.gshard[:valid].float(), valid)
                    with torch.no_grad():
                        p_slice.copy_(b.master[:valid])
            if self.dp.enabled:
                mine = b.param[lo : lo + b.slice]
                if cuda:
                    dist.all_gather_into_tensor(b.param, mine, group=self.dp.group)  # in place
                else:
                    parts = [torch.empty_like(mine) for _ in range(self.dp.world)]
                    dist.all_gather(parts, mine.clone(), group=self.dp.group)
                    with torch.no_grad():
                        b.param.copy_(torch.cat(parts))

    def _adam(self, b: _Bucket, gv: torch.Tensor, valid: int) -> None:
        """Adam (PyTorch ops) on the first ``valid`` owned elements, fp32 gradient ``gv``."""
        beta1, beta2 = self.betas
        bc1 = 1 - beta1**self._step
        bc2 = 1 - beta2**self._step
        m, v, w = b.exp_avg[:valid], b.exp_avg_sq[:valid], b.master[:valid]
        if self.weight_decay:
            w.mul_(1 - self.lr * self.weight_decay)
        m.lerp_(gv, 1 - beta1)
        v.mul_(beta2).addcmul_(gv, gv, value=1 - beta2)
        denom = (v.sqrt() / (bc2**0.5)).add_(self.eps)
        w.addcdiv_(m, denom, value=-self.lr / bc1)

    def _launch_emulated(self, b: _Bucket) -> None:
        g = b.grad.float()
        if self.dp.enabled:
            dist.all_reduce(g, group=self.dp.group)
        lo = self.dp.rank * b.slice
        gs = g[lo : lo + b.slice] / self.dp.world
        valid = max(0, min(b.slice, b.numel - lo))
        self._adam(b, gs[:valid], valid)
        mine = b.master.to(self.dtype)
        if self.dp.enabled:
            parts = [torch.empty_like(mine) for _ in range(self.dp.world)]
            dist.all_gather(parts, mine, group=self.dp.group)
            full = torch.cat(parts)
        else:
            full = mine
        with torch.no_grad():
            b.param.copy_(full)

    # -- optimizer API ------------------------------------------------------
    def step(self) -> None:
        """Launch the buckets still pending (all of them for pipelines; the SP bucket
        after ``finalize_grads``) and make the compute stream wait for the updates."""
        for b in self.buckets:
            if not b.launched:
                for i in range(len(b.params)):
                    if b.late or i not in b.filled:
                        if not self.native:
                            b.stage(i)
                        b.filled.add(i)
        self._launch_ready_all()
        if self.native:
            if self.record_timings:
                ev_main = torch.cuda.Event(enable_timing=True)
                ev_main.record(torch.cuda.current_stream(self.device))
                ev_side = torch.cuda.Event(enable_timing=True)
                ev_side.record(self.side)
                self._tail = (ev_main, ev_side)
            torch.cuda.current_stream(self.device).wait_stream(self.side)
        for b in self.buckets:
            b.filled = set()
            b.launched = False
        self._next = 0
        self._stepped = False

    def _launch_ready_all(self) -> None:
        while self._next < len(self.buckets):
            self._launch(self.buckets[self._next])
            self._next += 1

    # -- timing -------------------------------------------------------------
    def timings(self) -> dict:
        """Per-bucket timing of the last step run with ``record_timings`` set
        (synchronises the device): for every bucket, the milliseconds from its
        gradients being staged on the compute stream to its update finishing on
        the side stream, and ``exposed_ms``, how long the compute stream's last
        work of the step ran before the side stream finished (the DP time that
        backward did not hide; 0 or less when it was hidden). Clears the record."""
        if not self._events:
            return {}
        torch.cuda.synchronize(self.device)
        rows = [{"bucket": i, "numel": n, "stage_to_done_ms": round(a.elapsed_time(b), 4)}
                for i, n, a, b in self._events]
        out = {"buckets": rows}
        if self._tail is not None:
            out["exposed_ms"] = round(self._tail[0].elapsed_time(self._tail[1]), 4)
        self._events, self._tail = [], None
        return out

    # -- protocol invariants ------------------------------------------------
    def protocol_errors(self) -> List[str]:
        """Host-side check of the NVLink signal protocol after the last step
        (synchronises the device): every rank's flag words must show, for
        every rank r of the group, ``ready[r] == written[r] == epoch`` (the
        number of bucket launches, identical on all ranks), and the status
        word must be clear. Returns the violations (empty when all hold);
        collective over the DP group when it has several ranks."""
        if self.transport != "peer":
            return []
        torch.cuda.synchronize(self.device)
        n = self.dp.world
        words = self.flags.local.view(torch.int32)[: 2 * 8].cpu().tolist()  # [kind][kMaxRanks] uint32 flags
        ready, written = words[0:n], words[8 : 8 + n]
        errs = []
        if any(v != self.epoch for v in ready + written):
            errs.append(f"rank {self.dp.rank}: ready {ready} / written {written} != epoch {self.epoch}")
        if self.dp.enabled:
            epochs = [None] * n
            dist.all_gather_object(epochs, self.epoch, group=self.dp.group)
            if len(set(epochs)) != 1:
                errs.append(f"epochs differ across ranks: {epochs}")
        status = int(native.lib().read_status(False))
        if status:
            errs.append(f"rank {self.dp.rank}: status word {status}")
        return errs

    # -- state access (checkpoints) ----------------------------------------
    def full_state(self, p) -> Optional[dict]:
        """Gather the full fp32 master / moments of parameter ``p`` (collective
        over the DP group; call on every rank in the same order)."""
        b, i = self._where[id(p)]
        out = {}
        for name, shard in (("master", b.master), ("exp_avg", b.exp_avg), ("exp_avg_sq", b.exp_avg_sq)):
            if self.dp.enabled:
                parts = [torch.empty_like(shard) for _ in range(self.dp.world)]
                dist.all_gather(parts, shard.contiguous(), group=self.dp.group)
                full = torch.cat(parts)
            else:
                full = shard
            o = b.offsets[i]
            out[name] = full[o : o + p.numel()].view_as(p).clone()
        return out

    def load_full_state(self, p, master, exp_avg, exp_avg_sq, step: int) -> None:
        """Install this rank's slice of a full fp32 master / moment tensor of ``p``
        (checkpoint loading; any DP layout)."""
        b, i = self._where[id(p)]
        lo, hi = self.dp.rank * b.slice, (self.dp.rank + 1) * b.slice
        o0, o1 = b.offsets[i], b.offsets[i] + p.numel()
        a, z = max(lo, o0), min(hi, o1)
        if a < z:
            for shard, full in ((b.master, master), (b.exp_avg, exp_avg), (b.exp_avg_sq, exp_avg_sq)):
                shard[a - lo : z - lo].copy_(full.reshape(-1)[a - o0 : z - o0].to(shard.device, shard.dtype))
        self._step = int(step)
