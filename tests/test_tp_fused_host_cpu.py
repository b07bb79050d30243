"""Host-side bookkeeping of the gather-mode TP GEMM, with the native library
and peer buffers replaced by fakes that do what the kernel does to the
per-row-block arrival counters: after every launch, each remote row block's
counter equals epoch * (K / 64) - also when a channel sees a smaller and then
a larger token count again (the kernel waits for exactly that value)."""

import torch

from dstraining_b200.ops import tp_fused
from dstraining_b200.parallel.topology import TPContext


class _FakePeerBuffer:
    closed = []

    def __init__(self, nbytes, ctx, device):
        self.local = torch.zeros(nbytes, dtype=torch.uint8)
        self.ptrs = [0] * ctx.world
        self.device = torch.device("cpu")
        self.nbytes = nbytes

    def view(self, dtype):
        return self.local.view(dtype)

    def close(self):
        _FakePeerBuffer.closed.append(self)


class _FakeLib:
    def __init__(self, tp):
        self.tp = tp
        self.waits = []

    def tp_gemm(self, shard, a_mn, w, w_mn, M, N, K, epi, mode, bufs, flags, done, rank, seq, epoch, gath=None,
                arrive=None, **kw):
        kchunks = K // 64
        blocks = -(-M // 128)
        t_loc_blocks = seq // self.tp.world // 128
        for mb in range(blocks):  # blocks of other ranks' shards: copied, then waited for
            if (mb % (seq // 128)) // t_loc_blocks != rank:
                arrive[mb] += kchunks
                self.waits.append(int(arrive[mb]) >= epoch * kchunks)
        return (torch.zeros(M, N),)


def test_arrival_counters_follow_the_epoch(monkeypatch):
    tp = TPContext(group=None, rank=0, world=2, ranks=(0, 1))
    fake = _FakeLib(tp)
    monkeypatch.setattr(tp_fused, "PeerBuffer", _FakePeerBuffer)
    monkeypatch.setattr(tp_fused.native, "lib", lambda: fake)
    monkeypatch.setattr(tp_fused, "_CHANNELS", {})
    w = torch.zeros(64, 128)
    for seq in (1024, 512, 1024, 256, 1024):  # tokens of one batch row: the channel is created at 1024
        x = torch.zeros(seq // 2, 128)
        tp_fused.ag_gemm(1, "qkv.fwd", tp, x, seq, w, False, 0)
    assert fake.waits and all(fake.waits)


def test_growing_channel_is_retired_after_the_group_is_quiet(monkeypatch):
    """A channel that must grow (a larger activation arrives) is dropped only
    after every rank's work is finished (device synchronised, group barrier),
    and its peer mappings (data and flags) are closed, before the new one is
    made."""
    tp = TPContext(group=None, rank=0, world=2, ranks=(0, 1))
    fake = _FakeLib(tp)
    events = []
    monkeypatch.setattr(tp_fused, "PeerBuffer", _FakePeerBuffer)
    monkeypatch.setattr(tp_fused.native, "lib", lambda: fake)
    monkeypatch.setattr(tp_fused, "_CHANNELS", {})
    monkeypatch.setattr(tp_fused, "_quiesce", lambda ctx, dev: events.append(("quiesce", len(_FakePeerBuffer.closed))))
    _FakePeerBuffer.closed = []
    w = torch.zeros(64, 128)
    tp_fused.ag_gemm(1, "qkv.fwd", tp, torch.zeros(256, 128), 512, w, False, 0)
    old = tp_fused._CHANNELS[(1, "qkv.fwd", (0, 1))]
    tp_fused.ag_gemm(1, "qkv.fwd", tp, torch.zeros(128, 128), 256, w, False, 0)  # fits: same channel
    assert tp_fused._CHANNELS[(1, "qkv.fwd", (0, 1))] is old and not events
    tp_fused.ag_gemm(1, "qkv.fwd", tp, torch.zeros(512, 128), 1024, w, False, 0)  # grows
    new = tp_fused._CHANNELS[(1, "qkv.fwd", (0, 1))]
    assert new is not old and new.nbytes > old.nbytes
    assert events == [("quiesce", 0)]  # quiet first, then the mappings are closed
    assert old.buf in _FakePeerBuffer.closed and old.flags in _FakePeerBuffer.closed
