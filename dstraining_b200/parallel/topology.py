"""Process grid: who talks to whom.

The grid is 3-D. Global rank r decomposes as

    r = pp_rank * (tp * dp) + dp_rank * tp + tp_rank

so a tensor-parallel group is a run of ``tp`` consecutive ranks (on one B200
box: eight GPUs that all sit on the same NVSwitch, so the choice only matters
across nodes), a data-parallel group strides by ``tp`` inside one pipeline
stage, and pipeline neighbours stride by ``tp * dp``. The same layout as the
reference (``dst/parallel.py:134-172``); it is part of the public contract
because checkpoints and the data sampler key on it.

Contexts are frozen value objects; layers receive them at construction and
never consult global state, so a model built with :data:`SINGLE` is a plain
single-process model (the oracle every correctness test compares against).
"""

from __future__ import annotations

import datetime
import os
import sys
from dataclasses import dataclass, field
from typing import Optional, Tuple

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class TPContext:
    """One tensor-parallel (or data-parallel) group as seen from one rank.

    ``group`` is the process group (``None`` when ``world == 1``), ``rank``
    this process's index inside it, ``world`` its size. ``ranks`` lists the
    global ranks of the group in group order; the native peer-memory runtime
    uses it to map group slots to devices.
    """

    group: Optional[object]
    rank: int
    world: int
    ranks: Tuple[int, ...] = field(default=(0,), compare=False)

    @property
    def enabled(self) -> bool:
        return self.world > 1


SINGLE = TPContext(group=None, rank=0, world=1)


@dataclass(frozen=True)
class PPContext:
    """This rank's pipeline stage and its neighbours, as GLOBAL ranks.

    ``prev_rank``/``next_rank`` are ``None`` at the ends of the line;
    ``ring_prev_rank``/``ring_next_rank`` wrap around (the interleaved
    schedule moves activations on a ring).
    """

    rank: int
    world: int
    prev_rank: Optional[int]
    next_rank: Optional[int]
    ring_prev_rank: int = 0
    ring_next_rank: int = 0

    @property
    def is_first(self) -> bool:
        return self.rank == 0

    @property
    def is_last(self) -> bool:
        return self.rank == self.world - 1


PP_SINGLE = PPContext(rank=0, world=1, prev_rank=None, next_rank=None)

# A data-parallel group carries the same (group, rank, world) triple.
DPContext = TPContext
DP_SINGLE = SINGLE


def _pg_timeout() -> datetime.timedelta:
    # A short, configurable collective timeout is the host-side half of
    # failure detection: a rank that dies or stalls turns its peers' next
    # collective into an error instead of an indefinite wait.
    secs = float(os.environ.get("DST_PG_TIMEOUT_S", "600"))
    return datetime.timedelta(seconds=secs)


def init_distributed(backend: Optional[str] = None, timeout_s: Optional[float] = None) -> None:
    """Join the process group described by the launcher's environment.

    NCCL when CUDA is present, gloo otherwise; the code above this layer is
    identical for both, which is what lets every correctness suite run as
    CPU processes. ``DST_INIT_METHOD`` (e.g. ``file:///tmp/store``) selects a
    FileStore rendezvous with ``RANK``/``WORLD_SIZE`` from the environment;
    otherwise torchrun's ``MASTER_ADDR``/``MASTER_PORT`` are used. The device
    is bound from ``LOCAL_RANK`` before the first collective. Behaviour of
    the reference's ``dst/parallel.py:69-97``.
    """
    if dist.is_initialized():
        return
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "gloo" and sys.platform == "darwin":
        os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo0")
    timeout = datetime.timedelta(seconds=timeout_s) if timeout_s else _pg_timeout()
    if torch.cuda.is_available() and backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local % torch.cuda.device_count())
    kwargs = dict(backend=backend, timeout=timeout)
    init_method = os.environ.get("DST_INIT_METHOD")
    if init_method:
        kwargs.update(
            init_method=init_method,
            rank=int(os.environ["RANK"]),
            world_size=int(os.environ["WORLD_SIZE"]),
        )
    if backend == "nccl" and torch.cuda.is_available():
        # Binding the communicator to the device lets NCCL create it eagerly.
        kwargs["device_id"] = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group(**kwargs)


def default_device() -> torch.device:
    """CUDA device of this process when CUDA is available, else CPU (``dst/parallel.py:100-103``)."""
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _world() -> Tuple[int, int]:
    if not dist.is_initialized():
        return 0, 1
    return dist.get_rank(), dist.get_world_size()


def make_tp_context(tp_size: Optional[int] = None) -> TPContext:
    """Split the world into TP groups of consecutive ranks.

    ``dist.new_group`` is collective over the whole world, so every rank
    creates every group and keeps the one it belongs to.
    """
    rank, world = _world()
    tp_size = world if tp_size is None else tp_size
    if tp_size < 1 or world % tp_size:
        raise ValueError(f"world size {world} not divisible by tp size {tp_size}")
    if tp_size == 1:
        return SINGLE
    mine = None
    for base in range(0, world, tp_size):
        members = tuple(range(base, base + tp_size))
        pg = dist.new_group(list(members))
        if rank in members:
            mine = TPContext(group=pg, rank=rank - base, world=tp_size, ranks=members)
    assert mine is not None
    return mine


def grid_coords(rank: int, tp_size: int, pp_size: int, dp_size: int) -> Tuple[int, int, int]:
    """(tp_rank, pp_rank, dp_rank) of a global rank."""
    del pp_size
    stage_width = tp_size * dp_size
    return rank % tp_size, rank // stage_width, (rank // tp_size) % dp_size


def grid_rank(tp_rank: int, pp_rank: int, dp_rank: int, tp_size: int, dp_size: int) -> int:
    """Inverse of :func:`grid_coords`."""
    return pp_rank * tp_size * dp_size + dp_rank * tp_size + tp_rank


def make_topology(tp_size: int = 1, pp_size: int = 1, dp_size: int = 1):
    """Build the (tp, pp, dp) contexts of this rank."""
    rank, world = _world()
    if tp_size * pp_size * dp_size != world:
        raise ValueError(f"tp {tp_size} * pp {pp_size} * dp {dp_size} != world {world}")
    tp = make_tp_context(tp_size)
    tp_rank, pp_rank, dp_rank = grid_coords(rank, tp_size, pp_size, dp_size)

    def at_stage(stage: int) -> int:
        return grid_rank(tp_rank, stage, dp_rank, tp_size, dp_size)

    pp = PPContext(
        rank=pp_rank,
        world=pp_size,
        prev_rank=at_stage(pp_rank - 1) if pp_rank > 0 else None,
        next_rank=at_stage(pp_rank + 1) if pp_rank + 1 < pp_size else None,
        ring_prev_rank=at_stage((pp_rank - 1) % pp_size),
        ring_next_rank=at_stage((pp_rank + 1) % pp_size),
    )
    if dp_size == 1:
        return tp, pp, DP_SINGLE
    dp = None
    for s in range(pp_size):
        for t in range(tp_size):
            members = tuple(grid_rank(t, s, d, tp_size, dp_size) for d in range(dp_size))
            pg = dist.new_group(list(members))
            if rank in members:
                dp = DPContext(group=pg, rank=dp_rank, world=dp_size, ranks=members)
    assert dp is not None
    return tp, pp, dp


# ---------------------------------------------------------------- peer memory
_PEER_OK = {}  # group ranks -> bool


def _host_id() -> str:
    """This machine: host name plus the kernel's boot id (host names alone can
    repeat across containers on different machines)."""
    import socket

    boot = ""
    try:
        with open("/proc/sys/kernel/random/boot_id") as f:
            boot = f.read().strip()
    except OSError:
        pass
    return f"{socket.gethostname()}/{boot}"


def _pci_id(index: int) -> str:
    p = torch.cuda.get_device_properties(index)
    return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}"


def peers_addressable(infos, me: int, visible, can_access) -> bool:
    """Decision behind :func:`peer_reachable`, on the gathered facts.

    ``infos[r]`` is rank r's ``(host id, PCI id of its GPU)``; ``visible``
    maps the PCI ids of the GPUs this process can see to their device
    indices; ``can_access(a, b)`` answers whether device a can address
    device b's memory directly. True when every rank runs on this host, on a
    distinct GPU that this process sees and can address."""
    host, pci = infos[me]
    if pci not in visible or len({i[1] for i in infos}) != len(infos):
        return False
    mine = visible[pci]
    for r, (h, p) in enumerate(infos):
        if r == me:
            continue
        if h != host or p not in visible or not can_access(mine, visible[p]):
            return False
    return True


def peer_reachable(ctx: TPContext) -> bool:
    """Whether the peer-memory kernels (the fused DP optimizer and the fused
    tensor-parallel GEMMs, which load and store other ranks' buffers through
    CUDA IPC mappings) can serve this group: every rank on this host, on a GPU
    that this process can address directly. Groups spanning machines, or
    processes that cannot see their peers' GPUs, use the NCCL paths instead.
    ``DST_PEER=0`` forces the NCCL paths.

    Collective over the group on the first call for a group (every member
    must make it at the same point); cached afterwards. Single-rank groups
    are trivially reachable."""
    if not ctx.enabled:
        return True
    key = tuple(ctx.ranks)
    if key in _PEER_OK:
        return _PEER_OK[key]
    ok = torch.cuda.is_available() and dist.is_initialized() and os.environ.get("DST_PEER", "1") != "0"
    if torch.cuda.is_available() and dist.is_initialized():
        # every member takes part in both gathers, whatever its own answer, and
        # the group uses peer memory only if every member can: all agree
        mine = (_host_id(), _pci_id(torch.cuda.current_device()))
        infos = [None] * ctx.world
        dist.all_gather_object(infos, mine, group=ctx.group)
        visible = {_pci_id(i): i for i in range(torch.cuda.device_count())}
        ok = ok and peers_addressable(infos, ctx.rank, visible, torch.cuda.can_device_access_peer)
        votes = [None] * ctx.world
        dist.all_gather_object(votes, bool(ok), group=ctx.group)
        if not all(votes) and ctx.rank == 0 and os.environ.get("DST_PEER", "1") != "0":
            import warnings

            warnings.warn(f"ranks {list(ctx.ranks)} cannot all address each other's GPU memory "
                          f"(hosts / GPUs: {infos}); this group uses NCCL instead of the peer-memory kernels")
        ok = all(votes)
    _PEER_OK[key] = bool(ok)
    return _PEER_OK[key]
