"""Per-kernel micro-benchmark for the native sm_100a kernels.

    python -m dstraining_b200.utils.kernel_bench --suite gpt2        # every GPT-2-small shape
    python -m dstraining_b200.utils.kernel_bench --op gemm --m 16384 --n 3072 --k 768 --layout nt --epi bias_gelu
    python -m dstraining_b200.utils.kernel_bench --op attn --b 16 --t 1024 --h 12 --d 64 --dir bwd
    python -m dstraining_b200.utils.kernel_bench --op tp_gather --tp 4   # fused TP GEMM, emulated on 1 GPU

Each measurement: ``--warmup`` untimed calls, then ``--iters`` calls each
timed alone with CUDA events on the launching stream, with a 256 MB buffer
written just before each call so L2 (126 MB) holds nothing useful (that
write also keeps the GPU busy while the host queues the call, so the host's
launch work stays outside the interval); reports the mean
time, achieved TFLOP/s (GEMM, attention) or GB/s (memory-bound kernels), and
the fraction of the measured peaks in ``MEASURED_PEAKS.json`` (cuBLAS bf16
burst and copy bandwidth) when that file exists. Used as the small, bounded
case for ncu captures.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["hbm_gbs"], "of measured"
    return 1590.0, 6650.0, "of fallback"


class Timer:
    def __init__(self):
        self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def run(self, fn, warmup, iters):
        for _ in range(warmup):
            fn()
        total = 0.0
        for _ in range(iters):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            # The flush keeps the GPU busy while the host queues the start
            # event and the measured call, so the interval holds the kernels'
            # device time and not the host's launch work (as in a training
            # step, where launches run ahead of the device).
            self.flush.fill_(1.0)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            total += s.elapsed_time(e)
        return total / iters


def bf(*shape):
    return torch.randn(*shape, device="cuda").to(torch.bfloat16)


def bench_gemm(t, m, n, k, layout, epi, warmup, iters):
    from dstraining_b200.ops import gemm as G

    a_mn, b_mn = {"nt": (False, False), "nn": (False, True), "tn": (True, True)}[layout]
    A = bf(k, m) if a_mn else bf(m, k)
    B = bf(k, n) if b_mn else bf(n, k)
    bias, aux, aux_out = bf(n), bf(m, n), torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    code = {"store": G.EPI_STORE, "bias": G.EPI_BIAS, "bias_gelu": G.EPI_BIAS_GELU, "bias_resid": G.EPI_BIAS_RESID, "splitk": -1,
            "dgelu": G.EPI_DGELU}[epi]
    if epi == "splitk":
        fn = lambda: G.weight_grad(A, B)  # noqa: E731
    else:
        fn = lambda: G.gemm(A, a_mn, B, b_mn, code, bias=bias if "bias" in epi else None,  # noqa: E731
                            aux=aux if epi in ("bias_resid", "dgelu") else None,
                            aux_out=aux_out if epi == "bias_gelu" else None)
    ms = t.run(fn, warmup, iters)
    return ms, 2.0 * m * n * k / (ms * 1e-3) / 1e12


def bench_attn(t, b, tl, h, d, direction, warmup, iters, mode=0):
    from dstraining_b200.ops import native

    from dstraining_b200.ops.flash import padded_length

    lib = native.lib()
    if tl % 128:  # the model zero-pads such lengths up to the kernels' 128-row tiles
        tl = padded_length(tl)
    qkv = bf(b, tl, 3 * h * d)
    # mode 0: the model's dispatch; 1 / 2 force the ping-pong / one-tile forward
    fwd = lambda q, hh, dd: lib.flash_attn_fwd_tc(q, hh, dd, mode)  # noqa: E731
    out, lse = fwd(qkv, h, d)
    dout = bf(b, tl, h * d)
    if direction == "fwd":
        fn = lambda: fwd(qkv, h, d)  # noqa: E731
        flops = 4.0 * b * h * tl * tl * d / 2
    else:
        # mode 0: double-buffered kernels; 2: single-buffered
        fn = lambda: lib.flash_attn_bwd_tc(dout, qkv, out, lse, h, d, mode)  # noqa: E731
        flops = 10.0 * b * h * tl * tl * d / 2  # dV, dK, dQ, dP + the recomputed S
    ms = t.run(fn, warmup, iters)
    return ms, flops / (ms * 1e-3) / 1e12


def bench_tp_local(t, kind, tp, tokens, hidden, ffn, seq, warmup, iters, precopied=False):
    """The fused TP GEMMs as rank 0 of an emulated group on ONE GPU (every
    "rank's" buffer local, every peer flag raised: no launch waits for
    another kernel; see utils/tp_emulate.py): the kernel's own structure
    without NVLink, small enough for ncu. ``kind``: ``gather`` (AG+GEMM) or
    ``scatter`` (GEMM+RS with the ordered slot reduction)."""
    from dstraining_b200.ops import native
    from dstraining_b200.utils.tp_emulate import GatherEmulation, ScatterEmulation

    em = (GatherEmulation if kind == "gather" else ScatterEmulation)(tp, tokens, hidden, ffn, seq)
    ms = t.run(em.run, warmup, iters)
    if kind == "gather" and precopied:
        # the GEMM part alone: blocks already copied (the set-up copies are timed too, so report the
        # kernel from a separate event pair)
        times = []
        for _ in range(iters):
            em.run(precopied=True)  # warm
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            em.gath.copy_(em.gathered())
            em.epoch += 1
            em.arrive.fill_(em.epoch * (hidden // 64))
            em.done[1] = (tp - 1) * ((tokens // 128) // tp) * (hidden // 64)
            em.epoch -= 1
            t.flush.fill_(1.0)
            s.record()
            em.run()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        print(f"precopied gather GEMM: {sum(times) / len(times):.4f} ms")
    assert native.lib().read_status(True) == 0, "device status word set"
    return ms, 2.0 * tokens * ffn * hidden / (ms * 1e-3) / 1e12


def bench_ln(t, rows, c, direction, warmup, iters):
    from dstraining_b200.ops import native

    lib = native.lib()
    x, w, b, dy = bf(rows, c), bf(c), bf(c), bf(rows, c)
    y, mean, rstd = lib.layernorm_fwd(x, w, b, 1e-5)
    if direction == "fwd":
        fn = lambda: lib.layernorm_fwd(x, w, b, 1e-5)  # noqa: E731
        nbytes = 2 * rows * c * 2
    else:
        fn = lambda: lib.layernorm_bwd(dy, x, w, mean, rstd)  # noqa: E731
        nbytes = 3 * rows * c * 2 + 2 * rows * c * 2  # dx pass + the dγ/dβ column pass
    ms = t.run(fn, warmup, iters)
    return ms, nbytes / (ms * 1e-3) / 1e9


def gpt2_suite(t, warmup, iters):
    tok, C, V = 16384, 768, 50304
    rows = []
    for name, (m, n, k, lay, epi) in {
        "qkv fwd": (tok, 3 * C, C, "nt", "bias"),
        "proj fwd (+resid)": (tok, C, C, "nt", "bias_resid"),
        "fc fwd (+gelu)": (tok, 4 * C, C, "nt", "bias_gelu"),
        "c_proj fwd (+resid)": (tok, C, 4 * C, "nt", "bias_resid"),
        "head fwd": (tok, V, C, "nt", "store"),
        "c_proj dX (+dgelu)": (tok, 4 * C, C, "nn", "dgelu"),
        "fc dX": (tok, C, 4 * C, "nn", "store"),
        "qkv dX": (tok, C, 3 * C, "nn", "store"),
        "head dX": (tok, C, V, "nn", "store"),
        "fc dW (split-K)": (4 * C, C, tok, "tn", "splitk"),
        "c_proj dW (split-K)": (C, 4 * C, tok, "tn", "splitk"),
        "qkv dW (split-K)": (3 * C, C, tok, "tn", "splitk"),
        "head dW": (V, C, tok, "tn", "store"),
    }.items():
        ms, tf = bench_gemm(t, m, n, k, lay, epi, warmup, iters)
        rows.append((name, f"{m}x{n}x{k}", ms, tf, "TFLOP/s"))
    for d in ("fwd", "bwd"):
        ms, tf = bench_attn(t, 16, 1024, 12, 64, d, warmup, iters)
        rows.append((f"attention {d}", "b16 t1024 h12 d64", ms, tf, "TFLOP/s"))
    for d in ("fwd", "bwd"):
        ms, gb = bench_ln(t, tok, C, d, warmup, iters)
        rows.append((f"layernorm {d}", f"{tok}x{C}", ms, gb, "GB/s"))
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--suite", choices=["gpt2"], default=None)
    ap.add_argument("--op", choices=["gemm", "attn", "ln", "tp_gather", "tp_scatter"], default="gemm")
    ap.add_argument("--tp", type=int, default=4, help="tp_gather / tp_scatter: emulated group size")
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--ffn", type=int, default=2048, help="per-rank FFN width")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--precopied", action="store_true",
                    help="tp_gather: also time the GEMM part alone (remote blocks copied beforehand)")
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--k", type=int, default=768)
    ap.add_argument("--layout", default="nt")
    ap.add_argument("--epi", default="store")
    ap.add_argument("--b", type=int, default=16)
    ap.add_argument("--t", type=int, default=1024)
    ap.add_argument("--h", type=int, default=12)
    ap.add_argument("--d", type=int, default=64)
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--c", type=int, default=768)
    ap.add_argument("--dir", default="fwd")
    ap.add_argument("--attn-mode", type=int, default=0,
                    help="forward: 0 auto, 1 ping-pong, 2 one tile per CTA; backward: 0 double-buffered, 2 single")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    t = Timer()
    tf_peak, gb_peak, tag = peaks()
    if a.suite == "gpt2":
        rows = gpt2_suite(t, a.warmup, a.iters)
    elif a.op == "gemm":
        ms, tf = bench_gemm(t, a.m, a.n, a.k, a.layout, a.epi, a.warmup, a.iters)
        rows = [(f"gemm {a.layout} {a.epi}", f"{a.m}x{a.n}x{a.k}", ms, tf, "TFLOP/s")]
    elif a.op in ("tp_gather", "tp_scatter"):
        ms, tf = bench_tp_local(t, a.op[3:], a.tp, a.tokens, a.hidden, a.ffn, a.seq, a.warmup, a.iters,
                                a.precopied)
        rows = [(f"{a.op} (1 GPU, tp={a.tp})", f"{a.tokens}x{a.ffn}x{a.hidden}", ms, tf, "TFLOP/s")]
    elif a.op == "attn":
        ms, tf = bench_attn(t, a.b, a.t, a.h, a.d, a.dir, a.warmup, a.iters, a.attn_mode)
        rows = [(f"attention {a.dir}", f"b{a.b} t{a.t} h{a.h} d{a.d}", ms, tf, "TFLOP/s")]
    else:
        ms, gb = bench_ln(t, a.rows, a.c, a.dir, a.warmup, a.iters)
        rows = [(f"layernorm {a.dir}", f"{a.rows}x{a.c}", ms, gb, "GB/s")]
    print(f"{'kernel':24s} {'shape':22s} {'ms':>8s} {'achieved':>10s}  fraction")
    for name, shape, ms, val, unit in rows:
        peak = tf_peak if unit == "TFLOP/s" else gb_peak
        print(f"{name:24s} {shape:22s} {ms:8.4f} {val:8.1f} {unit:7s} {val / peak:6.1%} {tag}")


if __name__ == "__main__":
    main()
