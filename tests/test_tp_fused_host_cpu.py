"""Host-side bookkeeping of the gather-mode TP GEMM, with the native library
and peer buffers replaced by fakes that do what the kernel does to the
per-row-block arrival counters: after every launch, each remote row block's
counter equals epoch * (K / 64) - also when a channel sees a smaller and then
a larger token count again (the kernel waits for exactly that value)."""

import torch

from dstraining_b200.ops import tp_fused
from dstraining_b200.parallel.topology import TPContext


class _FakePeerBuffer:
    def __init__(self, nbytes, ctx, device):
        self.local = torch.zeros(nbytes, dtype=torch.uint8)
        self.ptrs = [0] * ctx.world

    def view(self, dtype):
        return self.local.view(dtype)


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
