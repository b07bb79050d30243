"""Pipeline schedules: 1F1B and interleaved 1F1B (virtual stages).

Compute order is the classic one. 1F1B: ``min(p-1-s, m)`` warm-up forwards,
then one-forward-one-backward, then the cool-down backwards, so at most
``p - s`` microbatches are in flight (``dst/pipeline.py:125-176``).
Interleaved (Megatron): ``tnm = m v`` forward and backward steps, warm-up
``min(2 (p-1-r) + (v-1) p, tnm)``, forward step ``i`` runs chunk
``(i mod pv) div p`` and backward step ``i`` runs chunk ``v-1-(i mod pv) div
p`` (``dst/pipeline.py:257-330``); it needs ``m % p == 0``.

Communication is designed for NCCL, not ported from the reference:

* Every directed link and flow gets its own two-rank communicator: forward
  activations ``stage s -> s+1`` and gradients ``s+1 -> s`` (plus the ring
  wrap links of the interleaved schedule). A communicator therefore carries
  only sends on one side and only receives on the other, always in schedule
  order, so FIFO matching is exact without tags and a waiting receive can
  never sit in front of an unrelated send on the same NCCL stream. (The
  reference shares world-spanning channel groups between pipeline columns
  and blocks the host in ``recv``, which deadlocks interleaved x TP on NCCL,
  ``README.md:275-283``.)
* Nothing blocks the host. Each receive is posted right before the forward
  or backward that consumes it, and the compute stream (not the host) waits
  on it. Sends are fire-and-forget on the link's stream; their buffers are
  held until the end of ``train_step``. A receive is never outstanding
  before this rank has sent everything the peer needs to reach the matching
  send, so host-side synchronisation inside a step cannot close a cycle.
* Communicators are created and warmed (one blocking send/recv per link)
  once at construction, every rank visiting every link in one global order,
  so lazy NCCL communicator init can never interleave with schedule
  traffic.
* Kernels are loaded when the CUDA context is created
  (``CUDA_MODULE_LOADING=EAGER``, set by importing ``dstraining_b200``):
  with lazy loading the first launch of a kernel waits for the device to go
  idle, which a stage holding an outstanding send or receive, or a fused
  collective spinning on a peer's flag, may not do while its peer is stuck
  the same way.

Under sequence parallelism the boundary tensor is ``[mb, T/tp, C]``.
The last stage scales each microbatch loss by ``1/m``; ``train_step``
returns the sum of those scaled losses (the batch mean) on the last stage
and ``None`` elsewhere. Gradients accumulate on the stage's parameters.
"""

from __future__ import annotations

import os
import warnings
from collections import deque
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .topology import PPContext

_LINKS: Dict[Tuple[str, int, int], object] = {}


def _column_ranks(pp: PPContext) -> List[int]:
    """Global ranks of this rank's pipeline column, by stage."""
    me = dist.get_rank()
    if pp.world == 1:
        return [me]
    stride = (pp.next_rank - me) if pp.next_rank is not None else (me - pp.prev_rank)
    first = me - pp.rank * stride
    return [first + s * stride for s in range(pp.world)]


def _all_columns(pp: PPContext) -> List[List[int]]:
    """Every pipeline column of the world (needed because group creation is
    collective over the world)."""
    world = dist.get_world_size()
    stride = world // pp.world
    return [[c + s * stride for s in range(pp.world)] for c in range(stride)]


def _check_module_loading(device: torch.device) -> None:
    """Sends are fire-and-forget (a kernel spinning until the peer receives),
    so a kernel's first launch must not wait for the device to go idle (lazy
    module loading does)."""
    if device.type == "cuda" and os.environ.get("CUDA_MODULE_LOADING", "LAZY").upper() != "EAGER":
        warnings.warn(
            "CUDA_MODULE_LOADING is not EAGER: a pipeline stage may deadlock on its first step "
            "(set it before CUDA is initialised; importing dstraining_b200 first does this)",
            RuntimeWarning,
        )


def _build_links(pp: PPContext, ring: bool, device: torch.device) -> None:
    """Create (once per process) the two-rank link communicators for every
    column, in one global order, and warm the ones this rank belongs to."""
    _check_module_loading(device)
    p = pp.world
    me = dist.get_rank()
    hops = p if ring else p - 1
    new_keys = []
    for column in _all_columns(pp):
        for flow in ("fwd", "bwd"):
            for s in range(hops):
                a, b = column[s], column[(s + 1) % p]
                src, dst = (a, b) if flow == "fwd" else (b, a)
                key = (flow, src, dst)
                if key in _LINKS:
                    continue
                _LINKS[key] = dist.new_group(sorted({src, dst}))
                new_keys.append(key)
    # Every communicator exists before any traffic. Then one real send/recv
    # per link (not a collective), in the same global order everywhere, so
    # the p2p connection NCCL sets up per peer pair exists before a schedule
    # posts its first receive; each is completed before the next.
    warm = torch.zeros(1, device=device)
    for flow, src, dst in new_keys:
        g = _LINKS[(flow, src, dst)]
        if me == src:
            dist.send(warm, dst=dst, group=g)
        elif me == dst:
            dist.recv(warm, src=src, group=g)
        if warm.is_cuda and me in (src, dst):
            torch.cuda.current_stream().synchronize()


class _Link:
    """One directed flow between two global ranks: posts sends or receives
    in schedule order."""

    def __init__(self, flow: str, src: int, dst: int):
        self.group = _LINKS[(flow, src, dst)]
        self.src, self.dst = src, dst

    def isend(self, t: torch.Tensor, keep: list) -> None:
        t = t.detach().contiguous()
        keep.append((dist.isend(t, dst=self.dst, group=self.group), t))

    def irecv(self, shape, dtype, device) -> Tuple[object, torch.Tensor]:
        buf = torch.empty(shape, dtype=dtype, device=device)
        return dist.irecv(buf, src=self.src, group=self.group), buf


class _RecvQueue:
    """Receives for one incoming link, handed out in FIFO order. Each receive
    is posted when its tensor is needed (``depth`` = 0): a receive posted
    earlier is a kernel spinning on the device until the peer sends, and any
    device-wide synchronisation on this rank in the meantime (an allocator
    ``cudaFree``, a library handle's first use, an ``.item()``) would then
    wait for a send the peer can only make after this rank continues. The
    exposed transfer is one boundary tensor over NVLink (tens of
    microseconds)."""

    def __init__(self, link: Optional[_Link], count: int, shape, dtype, device, depth: int = 0):
        self.link, self.remaining = link, count
        self.shape, self.dtype, self.device, self.depth = shape, dtype, device, depth
        self.posted: deque = deque()
        self._top_up()

    def _top_up(self) -> None:
        while self.link is not None and self.remaining and len(self.posted) < self.depth:
            self.posted.append(self.link.irecv(self.shape, self.dtype, self.device))
            self.remaining -= 1

    def pop(self) -> torch.Tensor:
        if not self.posted and self.link is not None and self.remaining:
            self.posted.append(self.link.irecv(self.shape, self.dtype, self.device))
            self.remaining -= 1
        work, buf = self.posted.popleft()
        work.wait()  # NCCL: a stream wait, not a host block
        self._top_up()
        return buf


def order_1f1b(p: int, s: int, m: int) -> List[Tuple[str, int]]:
    """Op order of stage ``s`` of ``p`` for ``m`` micro-batches: ``("F", i)``
    runs micro-batch i forward, ``("B", i)`` backward. ``min(p - 1 - s, m)``
    warm-up forwards, then one forward and one backward alternately, then the
    remaining backwards (``dst/pipeline.py:138-171``)."""
    n_warm = min(p - 1 - s, m)
    ops = [("F", i) for i in range(n_warm)]
    for i in range(n_warm, m):
        ops += [("F", i), ("B", i - n_warm)]
    ops += [("B", i) for i in range(m - n_warm, m)]
    return ops


def interleaved_chunk(step: int, p: int, v: int, forward: bool) -> int:
    """Model chunk of the ``step``-th forward (backward) of a rank in the
    interleaved schedule: groups of ``p`` steps per chunk, chunks ascending
    forward and descending backward (``dst/pipeline.py:278-280``)."""
    c = (step % (p * v)) // p
    return c if forward else v - 1 - c


def order_interleaved(p: int, r: int, v: int, m: int) -> List[Tuple[str, int]]:
    """Op order of rank ``r`` of ``p`` with ``v`` chunks and ``m`` micro-batches:
    ``("F", k)`` is the rank's k-th forward step, ``("B", k)`` its k-th backward
    step (chunk from :func:`interleaved_chunk`). Warm-up depth
    ``min(2 (p - 1 - r) + (v - 1) p, m v)`` as in ``dst/pipeline.py:269-270``."""
    tnm = m * v
    n_warm = min(2 * (p - 1 - r) + (v - 1) * p, tnm)
    ops = [("F", i) for i in range(n_warm)]
    for j in range(tnm - n_warm):
        ops += [("F", n_warm + j), ("B", j)]
    ops += [("B", j) for j in range(tnm - n_warm, tnm)]
    return ops


def _param_meta(module) -> Tuple[torch.dtype, torch.device]:
    p0 = next(module.parameters())
    return p0.dtype, p0.device


class Pipeline1F1B:
    """1F1B pipeline schedule over a :class:`GPTStage` (``dst/pipeline.py:52-176``):
    ``train_step(idx, targets)`` runs ``batch / micro_batch_size`` microbatches and
    returns the batch-mean loss on the last stage (``None`` elsewhere);
    ``eval_step`` is the forward-only counterpart."""

    def __init__(self, stage, pp: PPContext, micro_batch_size: int, seq_len: int):
        cfg = stage.config
        self.stage, self.pp = stage, pp
        self.micro_batch_size = micro_batch_size
        t_local = seq_len // stage.tp.world if cfg.sequence_parallel else seq_len
        self.act_shape = (micro_batch_size, t_local, cfg.n_embd)
        self.act_dtype, self.act_device = _param_meta(stage)
        self.fwd_in = self.fwd_out = self.bwd_in = self.bwd_out = None
        if pp.world > 1:
            _build_links(pp, ring=False, device=self.act_device)
            col = _column_ranks(pp)
            s = pp.rank
            if s > 0:
                self.fwd_in = _Link("fwd", col[s - 1], col[s])
                self.bwd_out = _Link("bwd", col[s], col[s - 1])
            if s < pp.world - 1:
                self.fwd_out = _Link("fwd", col[s], col[s + 1])
                self.bwd_in = _Link("bwd", col[s + 1], col[s])

    def train_step(self, idx: torch.Tensor, targets: torch.Tensor):
        b = idx.shape[0]
        if b % self.micro_batch_size:
            raise ValueError(f"batch {b} not divisible by micro batch {self.micro_batch_size}")
        m = b // self.micro_batch_size
        p, s = self.pp.world, self.pp.rank
        micro_idx = idx.split(self.micro_batch_size)
        micro_tgt = targets.split(self.micro_batch_size)
        meta = (self.act_shape, self.act_dtype, self.act_device)
        fwd_q = _RecvQueue(self.fwd_in, m, *meta)
        bwd_q = _RecvQueue(self.bwd_in, m, *meta)
        sent: list = []
        losses: List[torch.Tensor] = []
        stash: deque = deque()

        def forward(i: int) -> None:
            if self.pp.is_first:
                inp, x = None, micro_idx[i]
            else:
                inp = fwd_q.pop().requires_grad_(True)
                x = inp
            if self.pp.is_last:
                _, loss = self.stage(x, micro_tgt[i])
                out = loss / m
                losses.append(out.detach())
            else:
                out = self.stage(x)
                self.fwd_out.isend(out, sent)
            stash.append((inp, out))

        def backward() -> None:
            inp, out = stash.popleft()
            grad = None if self.pp.is_last else bwd_q.pop()
            torch.autograd.backward(out, grad_tensors=grad)
            if inp is not None:
                self.bwd_out.isend(inp.grad, sent)

        for op, i in order_1f1b(p, s, m):
            if op == "F":
                forward(i)
            else:
                backward()  # micro-batches leave the stash in order: this is micro-batch i
        for work, _ in sent:
            work.wait()
        assert not stash
        return torch.stack(losses).sum() if self.pp.is_last else None

    def eval_step(self, idx: torch.Tensor, targets: torch.Tensor):
        """Forward-only pass over the microbatches (no stash, no backward): each
        stage receives, runs and sends in microbatch order. Returns the mean loss
        on the last stage, ``None`` elsewhere."""
        b = idx.shape[0]
        if b % self.micro_batch_size:
            raise ValueError(f"batch {b} not divisible by micro batch {self.micro_batch_size}")
        m = b // self.micro_batch_size
        meta = (self.act_shape, self.act_dtype, self.act_device)
        fwd_q = _RecvQueue(self.fwd_in, m, *meta)
        sent: list = []
        total = None
        with torch.no_grad():
            for x_i, y_i in zip(idx.split(self.micro_batch_size), targets.split(self.micro_batch_size)):
                x = x_i if self.pp.is_first else fwd_q.pop()
                if self.pp.is_last:
                    _, loss = self.stage(x, y_i)
                    total = loss / m if total is None else total + loss / m
                else:
                    self.fwd_out.isend(self.stage(x), sent)
            for work, _ in sent:
                work.wait()
        return total


class PipelineInterleaved:
    """Interleaved 1F1B over the ``v`` chunks of a :class:`GPTChunks`.
    ``peak_in_flight`` records the largest number of stashed (input, output)
    pairs seen, so tests can check the schedule stays bounded by its
    warm-up depth."""

    def __init__(self, model, pp: PPContext, micro_batch_size: int, seq_len: int):
        cfg = model.config
        self.model, self.pp, self.v = model, pp, model.v
        self.micro_batch_size = micro_batch_size
        t_local = seq_len // model.tp.world if cfg.sequence_parallel else seq_len
        self.act_shape = (micro_batch_size, t_local, cfg.n_embd)
        self.act_dtype, self.act_device = _param_meta(model)
        self.peak_in_flight = 0
        self.fwd_in = self.fwd_out = self.bwd_in = self.bwd_out = None
        p, r = pp.world, pp.rank
        if p > 1:
            _build_links(pp, ring=True, device=self.act_device)
            col = _column_ranks(pp)
            prev, nxt = col[(r - 1) % p], col[(r + 1) % p]
            self.fwd_in = _Link("fwd", prev, col[r])
            self.fwd_out = _Link("fwd", col[r], nxt)
            self.bwd_in = _Link("bwd", nxt, col[r])
            self.bwd_out = _Link("bwd", col[r], prev)

    def _is_vfirst(self, c: int) -> bool:
        return self.pp.rank == 0 and c == 0

    def _is_vlast(self, c: int) -> bool:
        return self.pp.rank == self.pp.world - 1 and c == self.v - 1

    def train_step(self, idx: torch.Tensor, targets: torch.Tensor):
        b = idx.shape[0]
        if b % self.micro_batch_size:
            raise ValueError(f"batch {b} not divisible by micro batch {self.micro_batch_size}")
        m = b // self.micro_batch_size
        p, r, v = self.pp.world, self.pp.rank, self.v
        if m % p:
            raise ValueError(f"interleaving needs microbatches {m} divisible by stages {p}")
        micro_idx = idx.split(self.micro_batch_size)
        micro_tgt = targets.split(self.micro_batch_size)
        tnm = m * v

        def chunk(step: int, forward: bool) -> int:
            return interleaved_chunk(step, p, v, forward)

        # Messages each incoming link will deliver, in order: one per forward
        # (backward) step whose chunk is not virtual-first (virtual-last).
        n_fwd_in = sum(1 for i in range(tnm) if not self._is_vfirst(chunk(i, True)))
        n_bwd_in = sum(1 for i in range(tnm) if not self._is_vlast(chunk(i, False)))
        meta = (self.act_shape, self.act_dtype, self.act_device)
        fwd_q = _RecvQueue(self.fwd_in if p > 1 else None, n_fwd_in if p > 1 else 0, *meta)
        bwd_q = _RecvQueue(self.bwd_in if p > 1 else None, n_bwd_in if p > 1 else 0, *meta)
        sent: list = []
        losses: List[torch.Tensor] = []
        stash = [deque() for _ in range(v)]
        fed = 0
        tgt = 0
        # With p == 1 the "ring" is this rank: activations pass between chunks
        # in memory.
        local_fwd: deque = deque()
        local_bwd: deque = deque()

        def fwd(step: int) -> None:
            nonlocal fed, tgt
            c = chunk(step, True)
            if self._is_vfirst(c):
                inp, x = None, micro_idx[fed]
                fed += 1
            else:
                src = fwd_q.pop() if p > 1 else local_fwd.popleft()
                inp = src.detach().requires_grad_(True)
                x = inp
            if self._is_vlast(c):
                _, loss = self.model.chunks[c](x, micro_tgt[tgt])
                tgt += 1
                out = loss / m
                losses.append(out.detach())
            else:
                out = self.model.chunks[c](x)
                if p > 1:
                    self.fwd_out.isend(out, sent)
                else:
                    local_fwd.append(out.detach())
            stash[c].append((inp, out))
            self.peak_in_flight = max(self.peak_in_flight, sum(len(q) for q in stash))

        def bwd(step: int) -> None:
            c = chunk(step, False)
            inp, out = stash[c].popleft()
            if self._is_vlast(c):
                grad = None
            else:
                grad = bwd_q.pop() if p > 1 else local_bwd.popleft()
            torch.autograd.backward(out, grad_tensors=grad)
            if not self._is_vfirst(c):
                if p > 1:
                    self.bwd_out.isend(inp.grad, sent)
                else:
                    local_bwd.append(inp.grad)

        for op, k in order_interleaved(p, r, v, m):
            if op == "F":
                fwd(k)
            else:
                bwd(k)
        for work, _ in sent:
            work.wait()
        assert all(not q for q in stash) and fed in (0, m)
        return torch.stack(losses).sum() if self.pp.is_last else None

    def eval_step(self, idx: torch.Tensor, targets: torch.Tensor):
        """Forward-only pass of the interleaved schedule: every forward step in the
        training order (chunk ``(i mod pv) div p``), no backward. Returns the mean
        loss on the rank holding the last virtual stage, ``None`` elsewhere."""
        b = idx.shape[0]
        if b % self.micro_batch_size:
            raise ValueError(f"batch {b} not divisible by micro batch {self.micro_batch_size}")
        m = b // self.micro_batch_size
        p, v = self.pp.world, self.v
        if m % p:
            raise ValueError(f"interleaving needs microbatches {m} divisible by stages {p}")
        micro_idx = idx.split(self.micro_batch_size)
        micro_tgt = targets.split(self.micro_batch_size)
        tnm = m * v

        def chunk(step: int) -> int:
            return interleaved_chunk(step, p, v, True)

        n_fwd_in = sum(1 for i in range(tnm) if not self._is_vfirst(chunk(i)))
        meta = (self.act_shape, self.act_dtype, self.act_device)
        fwd_q = _RecvQueue(self.fwd_in if p > 1 else None, n_fwd_in if p > 1 else 0, *meta)
        local: deque = deque()
        sent: list = []
        total = None
        fed = tgt = 0
        with torch.no_grad():
            for i in range(tnm):
                c = chunk(i)
                if self._is_vfirst(c):
                    x = micro_idx[fed]
                    fed += 1
                else:
                    x = fwd_q.pop() if p > 1 else local.popleft()
                if self._is_vlast(c):
                    _, loss = self.model.chunks[c](x, micro_tgt[tgt])
                    tgt += 1
                    total = loss / m if total is None else total + loss / m
                else:
                    out = self.model.chunks[c](x)
                    if p > 1:
                        self.fwd_out.isend(out, sent)
                    else:
                        local.append(out)
            for work, _ in sent:
                work.wait()
        return total
