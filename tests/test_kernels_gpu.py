"""Numerics of every native sm_100a kernel against an fp32 PyTorch reference
of the same op (inputs rounded to bf16 first, so only the kernel's own
arithmetic is measured). Small and ragged shapes exercise the bounds paths.
"""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _lib():
    from dstraining_b200.ops import native

    return native.lib()


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


@pytest.fixture(autouse=True)
def _status(cuda):
    lib = _lib()
    lib.read_status(True)
    yield
    assert lib.read_status(True) == 0, "a kernel recorded a device-side error (bounded wait expired or bad argument)"


SHAPES = [(128, 256, 64), (296, 384, 200), (1024, 768, 768), (512, 2304, 768), (256, 50304 // 8, 128), (64, 128, 1024)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("layout", ["nt", "nn", "tn"])
def test_gemm_layouts(M, N, K, layout):
    from dstraining_b200.ops.gemm import gemm

    a_mn, b_mn = {"nt": (False, False), "nn": (False, True), "tn": (True, True)}[layout]
    A = _bf(K, M, seed=1) if a_mn else _bf(M, K, seed=1)
    B = _bf(K, N, seed=2) if b_mn else _bf(N, K, seed=2)
    ref = (A.float().t() if a_mn else A.float()) @ (B.float() if b_mn else B.float().t())
    out = gemm(A, a_mn, B, b_mn)
    assert out.shape == (M, N)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("epi", ["bias", "gelu", "resid", "dgelu"])
def test_gemm_epilogues(epi):
    from dstraining_b200.ops import gemm as G

    M, N, K = 384, 768, 256
    x, w, b = _bf(M, K, seed=3), _bf(N, K, scale=0.05, seed=4), _bf(N, seed=5)
    acc = x.float() @ w.float().t()
    if epi == "bias":
        out, ref = G.gemm(x, False, w, False, G.EPI_BIAS, bias=b), acc + b.float()
    elif epi == "gelu":
        pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        out = G.gemm(x, False, w, False, G.EPI_BIAS_GELU, bias=b, aux_out=pre)
        assert _rel(pre, acc + b.float()) < 1e-2
        ref = F.gelu(pre.float(), approximate="tanh")
    elif epi == "resid":
        r = _bf(M, N, seed=6)
        out, ref = G.gemm(x, False, w, False, G.EPI_BIAS_RESID, bias=b, aux=r), acc + b.float() + r.float()
    else:
        pre = _bf(M, N, seed=7)
        out = G.gemm(x, False, w, False, G.EPI_DGELU, aux=pre)
        xp = pre.float().requires_grad_(True)
        (gx,) = torch.autograd.grad(F.gelu(xp, approximate="tanh"), xp, acc)
        ref = gx
    assert _rel(out, ref) < 1.5e-2


@pytest.mark.parametrize("M,N,K", [(768, 768, 16384), (2304, 768, 4096), (3072, 768, 1000)])
def test_weight_grad_splitk(M, N, K):
    from dstraining_b200.ops.gemm import weight_grad

    dy, x = _bf(K, M, seed=8), _bf(K, N, seed=9)
    ref = dy.float().t() @ x.float()
    out = weight_grad(dy, x)
    assert _rel(out, ref) < 1e-2
    # deterministic: a second run is bitwise identical
    assert torch.equal(out, weight_grad(dy, x))


def test_colsum():
    from dstraining_b200.ops.gemm import bias_grad

    x = _bf(5000, 768, seed=10)
    assert _rel(bias_grad(x), x.float().sum(0)) < 1e-2


@pytest.mark.parametrize("C", [128, 768, 2048])
def test_layernorm(C):
    lib = _lib()
    x, w, b, dy = _bf(1000, C, seed=11), _bf(C, seed=12), _bf(C, seed=13), _bf(1000, C, seed=14)
    y, mean, rstd = lib.layernorm_fwd(x, w, b, 1e-5)
    xr = x.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    br = b.float().requires_grad_(True)
    yr = F.layer_norm(xr, (C,), wr, br, 1e-5)
    assert _rel(y, yr) < 1e-2
    dx, dw, db = lib.layernorm_bwd(dy, x, w, mean, rstd)
    yr.backward(dy.float())
    assert _rel(dx, xr.grad) < 2e-2
    assert _rel(dw, wr.grad) < 2e-2
    assert _rel(db, br.grad) < 2e-2
    dx2, dw2, db2 = lib.layernorm_bwd(dy, x, w, mean, rstd)
    assert torch.equal(dw, dw2) and torch.equal(db, db2)


def test_embedding():
    lib = _lib()
    V, P, C, B, T = 1000, 320, 768, 4, 256
    wte, wpe = _bf(V, C, seed=15), _bf(P, C, seed=16)
    idx = torch.randint(0, V, (B, T), device="cuda")
    out = lib.embedding_fwd(idx, wte, wpe, 64, 128)
    ref = (wte.float()[idx] + wpe.float()[:T][None])[:, 64:192]
    assert _rel(out, ref) < 1e-2
    dy = _bf(B, T, C, seed=17)
    dwte, dwpe = lib.embedding_bwd(dy, idx, V, P)
    rwte = torch.zeros(V, C, device="cuda").index_add_(0, idx.reshape(-1), dy.float().reshape(-1, C))
    assert _rel(dwte, rwte) < 1e-2
    assert _rel(dwpe[:T], dy.float().sum(0)) < 1e-2
    assert dwpe[T:].abs().max().item() == 0


def test_ids_outside_vocabulary_are_reported():
    """A token id or a target id outside the vocabulary is recorded in the
    status word (code 7); the embedding backward drops its rows instead of
    writing outside the table."""
    lib = _lib()
    V, P, C, B, T = 1000, 128, 256, 2, 128
    wte, wpe = _bf(V, C, seed=19), _bf(P, C, seed=20)
    idx = torch.randint(0, V, (B, T), device="cuda")
    idx[1, 5] = V + 3
    lib.embedding_fwd(idx, wte, wpe, 0, T)
    torch.cuda.synchronize()
    assert lib.read_status(True) == 7
    dy = _bf(B, T, C, seed=21)
    dwte, _ = lib.embedding_bwd(dy, idx, V, P)
    torch.cuda.synchronize()
    assert lib.read_status(True) == 7
    keep = (idx != V + 3).reshape(-1)
    rwte = torch.zeros(V, C, device="cuda").index_add_(0, idx.reshape(-1)[keep], dy.float().reshape(-1, C)[keep])
    assert _rel(dwte, rwte) < 1e-2
    tmax = torch.zeros(4, 3, device="cuda")
    tsum = torch.ones(4, 3, device="cuda")
    lib.ce_merge_tiles(tmax, tsum, torch.tensor([0, 5, 9, 2], device="cuda"), 10)
    torch.cuda.synchronize()
    assert lib.read_status(True) == 0
    lib.ce_merge_tiles(tmax, tsum, torch.tensor([0, 5, 10, 2], device="cuda"), 10)
    torch.cuda.synchronize()
    assert lib.read_status(True) == 7


def _ref_attention(qkv, H, D):
    B, T, _ = qkv.shape
    y = qkv.float().view(B, T, H, 3, D)
    q, k, v = (y[:, :, :, i].transpose(1, 2) for i in range(3))
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return o.transpose(1, 2).reshape(B, T, H * D)


def _ref_lse2(qkv, H, D):
    """Base-2 log-sum-exp of the causal scaled scores, [B, H, T] (what the
    forward kernels save for backward)."""
    B, T, _ = qkv.shape
    y = qkv.float().view(B, T, H, 3, D)
    q, k = y[:, :, :, 0].transpose(1, 2), y[:, :, :, 1].transpose(1, 2)
    s = (q @ k.transpose(-2, -1)) / D**0.5
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    return torch.logsumexp(s, -1) / math.log(2.0)


# T = 200 and 300: not multiples of the kernels' 128-row tiles, zero-padded by ops/flash.py
@pytest.mark.parametrize("B,T,H,D", [(2, 128, 4, 64), (2, 256, 2, 128), (1, 1024, 12, 64), (1, 2048, 2, 128),
                                     (2, 200, 4, 64), (1, 300, 2, 128)])
def test_flash_attention(B, T, H, D):
    from dstraining_b200.ops.flash import flash_attention

    qkv = _bf(B, T, 3 * H * D, seed=18).requires_grad_(True)
    out = flash_attention(qkv, H, D)
    qr = qkv.detach().float().requires_grad_(True)
    ref = _ref_attention(qr, H, D)
    assert _rel(out, ref) < 2e-2
    dout = _bf(B, T, H * D, seed=19)
    out.backward(dout)
    ref.backward(dout.float())
    g, gr = qkv.grad.float().view(B, T, H, 3, D), qr.grad.view(B, T, H, 3, D)
    for i, name in enumerate("qkv"):
        assert _rel(g[..., i, :], gr[..., i, :]) < 3e-2, name
    # deterministic backward
    qkv2 = qkv.detach().clone().requires_grad_(True)
    flash_attention(qkv2, H, D).backward(dout)
    assert torch.equal(qkv2.grad, qkv.grad)


def test_fused_head_ce():
    from dstraining_b200.ops.fused_head import fused_head_loss
    from dstraining_b200.parallel.topology import SINGLE

    N, C, V, real = 512, 256, 1024, 1000
    x = _bf(4, N // 4, C, seed=20).requires_grad_(True)
    w = _bf(V, C, scale=0.05, seed=21).requires_grad_(True)
    tgt = torch.randint(0, real, (4, N // 4), device="cuda")
    loss = fused_head_loss(x, w, tgt, SINGLE, real, False)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    logits = (xr @ wr.t())[..., :real]
    ref = F.cross_entropy(logits.reshape(-1, real), tgt.reshape(-1))
    assert abs(loss.item() - ref.item()) < 2e-2
    loss.backward()
    ref.backward()
    assert _rel(x.grad, xr.grad) < 3e-2
    assert _rel(w.grad, wr.grad) < 3e-2
    assert w.grad[real:].abs().max().item() == 0


def test_adam_matches_torch():
    from dstraining_b200.optim.precision import MasterWeightOptimizer

    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(n, device="cuda").to(torch.bfloat16)) for n in (10, 4096, 12345)]
    opt = MasterWeightOptimizer(ps, lr=1e-3)
    ref_master = [p.detach().float().clone().requires_grad_(True) for p in ps]
    ref = torch.optim.Adam(ref_master, lr=1e-3)
    for step in range(3):
        for p, rm in zip(ps, ref_master):
            g = torch.randn_like(p, dtype=torch.float32).to(torch.bfloat16)
            p.grad = g
            rm.grad = g.float()
        opt.step()
        ref.step()
    for p, m, rm in zip(ps, opt.master_params, ref_master):
        assert (m - rm).abs().max().item() < 1e-6
        assert torch.equal(p.data, m.to(torch.bfloat16))
    st = opt.inner.state[opt.master_params[0]]
    assert st["exp_avg"].dtype == torch.float32 and float(st["step"]) == 3


def test_adamw_matches_torch():
    """Decoupled weight decay in the native multi-tensor Adam equals torch.optim.AdamW."""
    from dstraining_b200.optim.precision import MasterWeightOptimizer

    torch.manual_seed(1)
    ps = [torch.nn.Parameter(torch.randn(n, device="cuda").to(torch.bfloat16)) for n in (10, 4096, 12345)]
    opt = MasterWeightOptimizer(ps, lr=1e-3, weight_decay=0.1, decoupled_weight_decay=True)
    assert opt._native and opt._native_supports()
    ref_master = [p.detach().float().clone().requires_grad_(True) for p in ps]
    ref = torch.optim.AdamW(ref_master, lr=1e-3, weight_decay=0.1)
    for step in range(3):
        for p, rm in zip(ps, ref_master):
            g = torch.randn_like(p, dtype=torch.float32).to(torch.bfloat16)
            p.grad = g
            rm.grad = g.float()
        opt.step()
        ref.step()
    for p, m, rm in zip(ps, opt.master_params, ref_master):
        assert (m - rm).abs().max().item() < 1e-6
        assert torch.equal(p.data, m.to(torch.bfloat16))


@pytest.mark.parametrize("B,T,H,D", [(2, 128, 4, 64), (1, 512, 3, 128), (2, 1024, 12, 64), (1, 2048, 2, 128)])
def test_flash_forward_tcgen05(B, T, H, D):
    """The tcgen05 forward matches the fp32 reference, including the saved
    base-2 log-sum-exp that backward consumes."""
    lib = _lib()
    qkv = _bf(B, T, 3 * H * D, seed=30)
    out, lse = lib.flash_attn_fwd_tc(qkv, H, D)
    ref = _ref_attention(qkv, H, D)
    assert _rel(out, ref) < 2e-2
    assert (lse - _ref_lse2(qkv, H, D)).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,T,H,D", [(2, 256, 4, 64), (1, 1024, 3, 128), (2, 1024, 12, 64), (1, 2048, 2, 128)])
@pytest.mark.parametrize("growing", [False, True])
def test_flash_forward_pingpong(B, T, H, D, growing):
    """Two-tile ping-pong forward (O in TMEM, thresholded rescaling) vs the
    fp32 reference and the one-tile kernel. ``growing`` scales keys up along
    the sequence so that row maxima keep rising and rescales happen."""
    lib = _lib()
    qkv = _bf(B, T, 3 * H * D, seed=31)
    if growing:
        ramp = torch.linspace(1.0, 6.0, T, device=qkv.device).view(1, T, 1, 1)
        v = qkv.view(B, T, H, 3, D).float()
        v[:, :, :, 1] *= ramp
        qkv = v.view(B, T, 3 * H * D).to(torch.bfloat16).contiguous()
    out, lse = lib.flash_attn_fwd_tc(qkv, H, D, 1)
    ref = _ref_attention(qkv, H, D)
    assert _rel(out, ref) < 2e-2
    out2, lse2 = lib.flash_attn_fwd_tc(qkv, H, D, 2)
    assert (lse - lse2).abs().max().item() < 2e-2
    assert _rel(out, out2) < 2e-2
    assert lib.read_status(True) == 0


@pytest.mark.parametrize("B,T,H,D", [(2, 128, 4, 64), (1, 512, 3, 128), (2, 1024, 12, 64), (1, 2048, 2, 128)])
@pytest.mark.parametrize("mode", [0, 2])
def test_flash_backward_tcgen05(B, T, H, D, mode):
    """tcgen05 backward (double-buffered kernels: mode 0; single-buffered:
    mode 2) vs the fp32 reference; bitwise deterministic across runs."""
    lib = _lib()
    qkv = _bf(B, T, 3 * H * D, seed=40)
    dout = _bf(B, T, H * D, seed=41)
    out, lse = lib.flash_attn_fwd_tc(qkv, H, D)
    g = lib.flash_attn_bwd_tc(dout, qkv, out, lse, H, D, mode)
    qr = qkv.float().requires_grad_(True)
    _ref_attention(qr, H, D).backward(dout.float())
    gv, gr = g.float().view(B, T, H, 3, D), qr.grad.view(B, T, H, 3, D)
    for i, name in enumerate("qkv"):
        assert _rel(gv[..., i, :], gr[..., i, :]) < 3e-2, name
    assert torch.equal(g, lib.flash_attn_bwd_tc(dout, qkv, out, lse, H, D, mode))
    assert lib.read_status(True) == 0


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tp_gather_gemm_emulated(tp):
    """The AG+GEMM kernel as rank 0 of a group of ``tp`` with every rank's
    shard local (no cross-kernel waits): remote row blocks copied through
    the copier's shared-memory tiles, own rows read in place; equal to the
    plain GEMM of the gathered input, twice in a row (the arrival counters
    and claim counter carry over between launches)."""
    from dstraining_b200.ops.gemm import gemm
    from dstraining_b200.utils.tp_emulate import GatherEmulation

    lib = _lib()
    em = GatherEmulation(tp, tokens=2 * 128 * tp * 2, hidden=256, ffn=384, seq=128 * tp * 2, seed=tp)
    ref = gemm(em.gathered(), False, em.w, False)
    for _ in range(2):
        out = em.run()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert lib.read_status(True) == 0


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tp_scatter_gemm_emulated(tp):
    """The GEMM+RS kernel and slot reduction as rank 0 of a group of ``tp``
    (other ranks' slots zero): rank 0's rows of the plain product, twice."""
    from dstraining_b200.ops.gemm import gemm
    from dstraining_b200.utils.tp_emulate import ScatterEmulation

    lib = _lib()
    em = ScatterEmulation(tp, tokens=2 * 128 * tp * 2, hidden=256, ffn=384, seq=128 * tp * 2, seed=tp)
    full = gemm(em.h, False, em.w, False)
    ref = full[em.own_rows()]
    for _ in range(2):
        out = em.run()
        torch.cuda.synchronize()
        assert _rel(out, ref) < 1e-2
    assert lib.read_status(True) == 0
