"""Tensor-parallel layers with the collective fused into the GEMM (CUDA bf16).

Every TP collective of the Megatron layer pair runs inside a tcgen05 GEMM
kernel over NVLink peer memory (``tp_gemm`` in ``csrc/gemm.cu``):

* gather (AG + GEMM): the sequence-sharded operand is TMA-loaded tile by tile
  straight from the owning rank's buffer - the column-parallel forward
  (``g``), the row-parallel dX (``ḡ`` backward), and the gathered operand of
  the weight-gradient GEMMs;
* scatter (GEMM + reduce-scatter): each 32-row output chunk is TMA-stored into
  the owning rank's receive slot as soon as it is computed; ``tp_reduce`` then
  sums the slots in rank order with the bias and residual - the row-parallel
  forward (``ḡ``) and the column-parallel dX (``g`` backward).

Without sequence parallelism (replicated activations) the all-reduces ``f̄``
and ``f``'s backward are the scatter GEMM + reduce followed by a peer
all-gather of the reduced shards (``tp_allgather``).

Each call site owns a :class:`_Channel`: a peer buffer for the shard (or the
receive slots), the cross-rank flag words and a launch epoch. Channels are
created lazily, in the same order on every rank of the group (the model runs
the same code on each), and grown when a larger activation arrives. The
kernels' flag protocol makes reusing a channel safe: a shard buffer is not
rewritten before every peer has read it, a receive slot is not rewritten
before its owner has drained it.
"""

from __future__ import annotations

from typing import Dict, Tuple

import torch
import torch.distributed as dist

from ..parallel.symm import PeerBuffer
from ..parallel.topology import TPContext, peer_reachable
from . import native
from .gemm import EPI_BIAS, EPI_BIAS_GELU, EPI_DGELU, EPI_STORE, bias_grad, gemm, weight_grad

EPI_PARTIAL_F32 = 5
EPI_CE_STATS = 6
MODE_GATHER_A, MODE_GATHER_B, MODE_SCATTER = 1, 2, 3


class _Channel:
    def __init__(self, tp: TPContext, device: torch.device, nbytes: int):
        self.tp = tp
        self.buf = PeerBuffer(nbytes, tp, device)
        self.flags = PeerBuffer(64 * 4, tp, device)
        self.done = torch.zeros(2, dtype=torch.int32, device=device)  # CTA-done and copy-claim counters
        self.epoch = 0
        self.nbytes = nbytes

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def view(self, numel: int) -> torch.Tensor:
        return self.buf.view(torch.bfloat16)[:numel]

    def retire(self) -> None:
        """Release this channel's memory safely (collective over the group): a
        peer's kernel may still be reading or writing this rank's buffers over
        NVLink, which freeing memory does not wait for, so every rank first
        finishes its own work on the device, then the group agrees that all
        have, then each rank unmaps its peers' buffers; the local buffers are
        freed when the last reference goes."""
        _quiesce(self.tp, self.buf.device)
        self.buf.close()
        self.flags.close()


def _quiesce(tp: TPContext, device: torch.device) -> None:
    """Every rank of ``tp`` has finished all work queued on its device."""
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    if tp.enabled and dist.is_initialized():
        dist.barrier(group=tp.group)
        if device.type == "cuda":
            torch.cuda.synchronize(device)


_CHANNELS: Dict[Tuple[int, str, Tuple[int, ...]], _Channel] = {}


def channel(owner: int, role: str, tp: TPContext, nbytes: int, device: torch.device) -> _Channel:
    """The channel of one call site, keyed by the owning layer (the id of its
    weight Parameter, captured in forward), a role and the group's ranks (an
    id can be reused by a later model in another group); created or grown
    collectively in program order. A channel that must grow is retired first
    (every rank's work on it finished, peers' mappings closed)."""
    key = (owner, role, tuple(tp.ranks))
    ch = _CHANNELS.get(key)
    if ch is None or ch.nbytes < nbytes:
        if ch is not None:
            del _CHANNELS[key]
            ch.retire()
        ch = _Channel(tp, device, nbytes)
        _CHANNELS[key] = ch
    return ch


def _flat(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1, t.shape[-1])


def _publish_shard(ch: _Channel, x2: torch.Tensor) -> torch.Tensor:
    """Copy this rank's shard into the channel's peer buffer."""
    dst = ch.view(x2.numel()).view_as(x2)
    dst.copy_(x2)
    return dst


def ag_gemm(owner, role, tp: TPContext, x_shard2: torch.Tensor, seq: int, w: torch.Tensor, w_mn: bool, epi: int,
            **kw):
    """AG_tokens(x_shard) . op(w)^T (gather mode, rows of operand A).

    Returns ``(results, gathered)``: the kernel's outputs (``[tokens, N]``
    first) and the gathered ``[tokens, K]`` input, which the kernel assembles
    locally while it computes (each remote byte crosses NVLink once) and which
    backward reuses. Extra keywords (bias, aux, targets, ce_col0, ce_valid)
    go to the kernel."""
    ch = channel(owner, role, tp, x_shard2.numel() * 2, x_shard2.device)
    shard = _publish_shard(ch, x_shard2)
    tokens = x_shard2.shape[0] * tp.world
    n = w.shape[1] if w_mn else w.shape[0]
    # Per 128-row block, the kernel counts the 64-column chunks copied into the
    # gather buffer and waits for epoch * (K / 64): the counters advance only in
    # launches that cover their block, so they are set to the channel's epoch
    # whenever the token count changes (stream-ordered after the last launch).
    kchunks = x_shard2.shape[1] // 64
    if getattr(ch, "arrive", None) is None:
        ch.arrive = torch.full((-(-tokens // 128),), ch.epoch * kchunks, dtype=torch.int32, device=x_shard2.device)
        ch.arrive_tokens = tokens
    elif ch.arrive_tokens != tokens:
        ch.arrive.fill_(ch.epoch * kchunks)
        ch.arrive_tokens = tokens
    gathered = torch.empty(tokens, x_shard2.shape[1], dtype=x_shard2.dtype, device=x_shard2.device)
    res = native.lib().tp_gemm(
        shard, False, w, w_mn, tokens, n, x_shard2.shape[1], epi, MODE_GATHER_A, ch.buf.ptrs, ch.flags.ptrs, ch.done,
        tp.rank, seq, ch.next_epoch(), gath=gathered, arrive=ch.arrive, **kw,
    )
    # Rows of this rank's own shard are read in place by the kernel; fill
    # them into the gathered copy for backward.
    t_loc = seq // tp.world
    g3 = gathered.view(-1, seq, gathered.shape[1])
    g3[:, tp.rank * t_loc : (tp.rank + 1) * t_loc].copy_(x_shard2.view(-1, t_loc, x_shard2.shape[1]))
    return res, gathered


def gemm_rs(owner, role, tp: TPContext, a2: torch.Tensor, seq: int, w: torch.Tensor, w_mn: bool,
            bias=None, resid2=None) -> torch.Tensor:
    """[tokens/tp, N] = RS_tokens(a . op(w)^T) + bias + resid (scatter mode + slot reduction)."""
    tokens = a2.shape[0]
    n = w.shape[1] if w_mn else w.shape[0]
    rows = tokens // tp.world
    ch = channel(owner, role, tp, tokens * n * 2, a2.device)
    lib = native.lib()
    epoch = ch.next_epoch()
    lib.tp_gemm(a2, False, w, w_mn, tokens, n, a2.shape[1], EPI_STORE, MODE_SCATTER, ch.buf.ptrs, ch.flags.ptrs,
                ch.done, tp.rank, seq, epoch)
    recv = ch.view(tokens * n).view(tp.world, rows, n)
    return lib.tp_reduce(recv, tp.world, bias, resid2, ch.flags.ptrs, ch.done, tp.rank, epoch)


def allgather_rows(owner, role, tp: TPContext, shard2: torch.Tensor, seq: int) -> torch.Tensor:
    """Sequence shards [tokens/tp, N] of every rank -> full [tokens, N]."""
    ch = channel(owner, role, tp, shard2.numel() * 2, shard2.device)
    _publish_shard(ch, shard2)
    return native.lib().tp_allgather(ch.buf.ptrs, shard2.shape[0], shard2.shape[1], seq, ch.flags.ptrs, ch.done,
                                     tp.rank, ch.next_epoch(), shard2)


# ---------------------------------------------------------------------- layers
class _ColumnTP(torch.autograd.Function):
    """Column-parallel linear under TP. sequence mode: x [B, T/tp, C] -> y
    [B, T, N/tp] via AG+GEMM; replicated: x [B, T, C] -> y (no forward comm)."""

    @staticmethod
    def forward(ctx, x, w, b, tp, mode):
        B, t = x.shape[0], x.shape[1]
        x2 = _flat(x.contiguous())
        if mode == "sequence":
            seq = t * tp.world
            res, xg = ag_gemm(id(w), "col.fwd", tp, x2, seq, w, False, EPI_BIAS if b is not None else EPI_STORE, bias=b)
            y = res[0]
        else:
            seq = t
            y = gemm(x2, False, w, False, EPI_BIAS if b is not None else EPI_STORE, bias=b)
            xg = x2
        ctx.save_for_backward(xg, w)  # the (gathered) input, for dW
        ctx.meta = (tp, mode, seq, b is not None, x.shape, id(w))
        return y.view(B, seq, w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        xg, w = ctx.saved_tensors
        tp, mode, seq, has_b, xshape, k = ctx.meta
        dy2 = _flat(dy.contiguous())
        db = bias_grad(dy2) if has_b else None
        if mode == "sequence":
            dx = gemm_rs(k, "col.bwd.rs", tp, dy2, seq, w, True).view(xshape)
        else:
            dx_shard = gemm_rs(k, "col.bwd.rs", tp, dy2, seq, w, True)
            dx = allgather_rows(k, "col.bwd.ag", tp, dx_shard, seq).view(xshape)
        dw = weight_grad(dy2, xg)
        return dx, dw, db, None, None


class _RowTP(torch.autograd.Function):
    """Row-parallel linear under TP: y = exit(x W^T) + bias (+ residual).
    sequence mode: GEMM + reduce-scatter -> [B, T/tp, N]; replicated: GEMM +
    reduce-scatter + all-gather -> [B, T, N]."""

    @staticmethod
    def forward(ctx, x, w, b, residual, tp, mode):
        B, T = x.shape[0], x.shape[1]
        x2 = _flat(x.contiguous())
        rows = x2.shape[0] // tp.world
        if mode == "sequence":
            r2 = _flat(residual.contiguous()) if residual is not None else None
            y = gemm_rs(id(w), "row.fwd.rs", tp, x2, T, w, False, bias=b, resid2=r2).view(B, T // tp.world, w.shape[0])
        else:
            r2 = None
            if residual is not None:
                tl = T // tp.world
                r2 = _flat(residual[:, tp.rank * tl : (tp.rank + 1) * tl].contiguous())
            shard = gemm_rs(id(w), "row.fwd.rs", tp, x2, T, w, False, bias=b, resid2=r2)
            y = allgather_rows(id(w), "row.fwd.ag", tp, shard, T).view(B, T, w.shape[0])
        ctx.save_for_backward(x2, w)
        ctx.meta = (tp, mode, T, b is not None, residual is not None, x.shape, id(w))
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        tp, mode, T, has_b, has_res, xshape, k = ctx.meta
        dres = dy if has_res else None
        dy2 = _flat(dy.contiguous())
        db = bias_grad(dy2) if has_b else None  # sequence mode: partial, summed by finalize_grads
        if mode == "sequence":
            res, dyg = ag_gemm(k, "row.bwd.dx", tp, dy2, T, w, True, EPI_STORE)
            dx = res[0].view(xshape)
            dw = weight_grad(dyg, x2)
        else:
            dx = gemm(dy2, False, w, True, EPI_STORE).view(xshape)
            dw = weight_grad(dy2, x2)
        return dx, dw, db, dres, None, None


class _MLPTP(torch.autograd.Function):
    """c_proj(gelu(c_fc(x))) + residual under TP with sequence parallelism:
    AG+GEMM(+bias+GELU) then GEMM+RS(+bias+residual); backward mirrors it
    with dGELU in the epilogue of the gathered c_proj dX GEMM."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, residual, tp):
        B, tl = x.shape[0], x.shape[1]
        T = tl * tp.world
        x2 = _flat(x.contiguous())
        res, xg = ag_gemm(id(w1), "mlp.fc.fwd", tp, x2, T, w1, False, EPI_BIAS_GELU, bias=b1)
        h, pre = res[0], res[1]
        r2 = _flat(residual.contiguous()) if residual is not None else None
        y = gemm_rs(id(w2), "mlp.proj.fwd", tp, h, T, w2, False, bias=b2, resid2=r2).view(B, tl, w2.shape[0])
        ctx.save_for_backward(xg, w1, pre, h, w2)
        ctx.meta = (tp, T, b1 is not None, b2 is not None, residual is not None, x.shape, id(w1), id(w2))
        return y

    @staticmethod
    def backward(ctx, dy):
        xg, w1, pre, h, w2 = ctx.saved_tensors
        tp, T, has_b1, has_b2, has_res, xshape, k1, k2 = ctx.meta
        dres = dy if has_res else None
        dy2 = _flat(dy.contiguous())
        db2 = bias_grad(dy2) if has_b2 else None  # partial over the sequence shard
        res, dyg = ag_gemm(k2, "mlp.proj.bwd.dx", tp, dy2, T, w2, True, EPI_DGELU, aux=pre)
        dpre = res[0]
        dw2 = weight_grad(dyg, h)
        dx = gemm_rs(k1, "mlp.fc.bwd.rs", tp, dpre, T, w1, True).view(xshape)
        dw1 = weight_grad(dpre, xg)
        db1 = bias_grad(dpre) if has_b1 else None
        return dx, dw1, db1, dw2, db2, dres, None


class _MLPTPReplicated(torch.autograd.Function):
    """c_proj(gelu(c_fc(x))) + residual under TP without sequence parallelism
    (activations replicated): c_fc with its bias + GELU epilogue needs no
    communication; c_proj's all-reduce (f̄) is the scatter GEMM + ordered slot
    reduction (bias, residual) + peer all-gather of the reduced rows. Backward:
    dGELU in the epilogue of the local c_proj dX GEMM, and c_fc's dX all-reduce
    (f's backward) as scatter GEMM + reduction + all-gather."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2, residual, tp):
        B, T = x.shape[0], x.shape[1]
        x2 = _flat(x.contiguous())
        pre = torch.empty(x2.shape[0], w1.shape[0], dtype=x2.dtype, device=x2.device)
        h = gemm(x2, False, w1, False, EPI_BIAS_GELU, bias=b1, aux_out=pre)
        r2 = None
        if residual is not None:
            tl = T // tp.world
            r2 = _flat(residual[:, tp.rank * tl : (tp.rank + 1) * tl].contiguous())
        shard = gemm_rs(id(w2), "mlp.rep.proj.rs", tp, h, T, w2, False, bias=b2, resid2=r2)
        y = allgather_rows(id(w2), "mlp.rep.proj.ag", tp, shard, T).view(B, T, w2.shape[0])
        ctx.save_for_backward(x2, w1, pre, h, w2)
        ctx.meta = (tp, T, b1 is not None, b2 is not None, residual is not None, x.shape, id(w1))
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, w1, pre, h, w2 = ctx.saved_tensors
        tp, T, has_b1, has_b2, has_res, xshape, k1 = ctx.meta
        dres = dy if has_res else None
        dy2 = _flat(dy.contiguous())
        db2 = bias_grad(dy2) if has_b2 else None  # dy is replicated: complete on every rank
        dpre = gemm(dy2, False, w2, True, EPI_DGELU, aux=pre)
        dw2 = weight_grad(dy2, h)
        dx_shard = gemm_rs(k1, "mlp.rep.fc.bwd.rs", tp, dpre, T, w1, True)
        dx = allgather_rows(k1, "mlp.rep.fc.bwd.ag", tp, dx_shard, T).view(xshape)
        dw1 = weight_grad(dpre, x2)
        db1 = bias_grad(dpre) if has_b1 else None
        return dx, dw1, db1, dw2, db2, dres, None


def mlp_replicated(x, w1, b1, w2, b2, residual, tp):
    return _MLPTPReplicated.apply(x, w1, b1, w2, b2, residual, tp)


def column_parallel(x, w, b, tp, mode):
    return _ColumnTP.apply(x, w, b, tp, mode)


def row_parallel(x, w, b, residual, tp, mode):
    return _RowTP.apply(x, w, b, residual, tp, mode)


def mlp_sequence_parallel(x, w1, b1, w2, b2, residual, tp):
    return _MLPTP.apply(x, w1, b1, w2, b2, residual, tp)


def usable(tp: TPContext, seq: int) -> bool:
    """The fused kernels need sequence shards of a multiple of 128 tokens and
    a group whose ranks can address each other's GPU memory (one host; the
    first call per group is a collective, see ``peer_reachable``)."""
    return (tp.enabled and tp.world <= 8 and seq % tp.world == 0 and (seq // tp.world) % 128 == 0
            and peer_reachable(tp))
