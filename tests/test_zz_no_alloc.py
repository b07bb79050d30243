"""The allocation-free C entry point ``dst_layernorm_bwd_noalloc``.

It exists for callers that cannot allocate device memory themselves (a
plugin whose host runtime owns the memory pool, or a latency-critical path
that cannot afford cudaMalloc's device synchronisation); its scratch space is
a fixed array inside the library. This test calls it through its exported C
symbol, exactly as such a caller would, and checks it against the library's
regular (allocating) LayerNorm backward on two calls in a row - the second
call reuses the scratch array the first one left behind. The file is named so
pytest collects it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DST_NOALLOC_OK = 0
DST_NOALLOC_ERR_TOO_LARGE = 1
DST_NOALLOC_ERR_BAD_ARG = 2


def _entry():
    from dstraining_b200.ops import native

    lib = native.lib()
    so = ctypes.CDLL(lib.__file__)
    fn = so.dst_layernorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return lib, fn


def _call(fn, dy, x, w, mean, rstd, dx, dw, db, rows, hidden):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(
        dy.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
        dx.data_ptr(), dw.data_ptr(), db.data_ptr(), rows, hidden, stream,
    )


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


# 768 and 1024 take the two-kernel path; 1032 and up the three-kernel path,
# up to the largest accepted hidden size (DST_NOALLOC_MAX_HIDDEN = 4096).
@pytest.mark.parametrize("rows,hidden", [(3000, 768), (257, 1024), (300, 1032), (517, 2048), (1000, 3072), (333, 4096)])
def test_noalloc_matches_allocating_layernorm_bwd(cuda, rows, hidden):
    lib, fn = _entry()
    for call in range(2):  # two calls in a row share the scratch array
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        x = torch.randn(rows, hidden, device="cuda", generator=g).to(torch.bfloat16)
        w = torch.randn(hidden, device="cuda", generator=g).to(torch.bfloat16)
        b = torch.randn(hidden, device="cuda", generator=g).to(torch.bfloat16)
        dy = torch.randn(rows, hidden, device="cuda", generator=g).to(torch.bfloat16)
        _, mean, rstd = lib.layernorm_fwd(x, w, b, 1e-5)
        dx_ref, dw_ref, db_ref = lib.layernorm_bwd(dy, x, w, mean, rstd)
        dx = torch.empty_like(x)
        dw = torch.empty_like(w)
        db = torch.empty_like(w)
        assert _call(fn, dy, x, w, mean, rstd, dx, dw, db, rows, hidden) == DST_NOALLOC_OK
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 2e-2
        assert _rel(dw, dw_ref) < 2e-2
        assert _rel(db, db_ref) < 2e-2


def test_noalloc_rejects_oversized_and_bad_arguments(cuda):
    _, fn = _entry()
    rows, hidden = 16, 8192  # above DST_NOALLOC_MAX_HIDDEN (4096)
    t = torch.zeros(rows, hidden, device="cuda", dtype=torch.bfloat16)
    v = torch.zeros(hidden, device="cuda", dtype=torch.bfloat16)
    s = torch.zeros(rows, device="cuda")
    assert _call(fn, t, t, v, s, s, t, v, v, rows, hidden) == DST_NOALLOC_ERR_TOO_LARGE
    assert _call(fn, t, t, v, s, s, t, v, v, rows, 12) == DST_NOALLOC_ERR_BAD_ARG
    assert _call(fn, t, t, v, s, s, t, v, v, 0, 64) == DST_NOALLOC_ERR_BAD_ARG
    # dy, x, w and dx must start on a 16-byte boundary: an offset view is
    # refused instead of faulting inside the kernel.
    off = t.view(-1)[1:].view(-1)
    assert _call(fn, off, t, v, s, s, t, v, v, 2, 64) == DST_NOALLOC_ERR_BAD_ARG
    assert _call(fn, t, t, v, s, s, off, v, v, 2, 64) == DST_NOALLOC_ERR_BAD_ARG
