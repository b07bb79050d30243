"""Device-side failure detection: every cross-rank wait inside a kernel is
bounded. A peer flag that nothing ever sets makes the wait run out; the
kernel records a timeout in the status word and returns normally, and the
device stays usable. No fault, trap or hang is involved."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

K_TIMEOUT_PEER = 5


def test_bounded_peer_wait_reports_timeout(cuda):
    from dstraining_b200.ops import native

    lib = native.lib()
    lib.read_status(True)
    n = 4096
    # Two "ranks", both backed by buffers of this one GPU; rank 1 never runs,
    # so its "ready" flag never arrives.
    grads = [torch.zeros(2 * n, dtype=torch.bfloat16, device=cuda) for _ in range(2)]
    params = [torch.zeros(2 * n, dtype=torch.bfloat16, device=cuda) for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int32, device=cuda) for _ in range(2)]
    master, m, v = (torch.zeros(n, device=cuda) for _ in range(3))
    done = torch.zeros(1, dtype=torch.int32, device=cuda)
    t0 = time.time()
    lib.fused_dp_adam([g.data_ptr() for g in grads], [p.data_ptr() for p in params], [f.data_ptr() for f in flags],
                      master, m, v, done, n, 2 * n, 0, 1, 1e-3, 0.9, 0.999, 1e-8, 1.0)
    status = lib.read_status(True)  # synchronises
    elapsed = time.time() - t0
    assert status == K_TIMEOUT_PEER
    assert elapsed < 30
    assert master.abs().max().item() == 0  # the update was skipped, not half-applied
    # the context is healthy: a normal kernel still runs and is correct
    a = torch.randn(256, 128, device=cuda).to(torch.bfloat16)
    b = torch.randn(128, 128, device=cuda).to(torch.bfloat16)
    out = lib.gemm(a, False, b, False, 0)
    ref = a.float() @ b.float().t()
    assert ((out.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2  # bf16 output rounding
    assert lib.read_status(True) == 0
