"""Fused compute+collective kernels vs the NCCL baseline, per rank.

    torchrun --nproc-per-node N -m dstraining_b200.utils.comm_bench [--tokens 8192 --hidden 2048]

One process per GPU. Times, with CUDA events on the launching stream (after
warm-up, synchronised on both sides, max over ranks):

* AG+GEMM  (column-parallel forward, sequence-sharded input):
  fused ``tp_gemm`` gather mode  vs  NCCL all_gather_into_tensor + GEMM
* GEMM+RS  (row-parallel forward):
  fused scatter mode + slot reduction  vs  GEMM + NCCL reduce_scatter_tensor
* DP bucket step (25 MiB bf16 bucket):
  fused reduce + sharded Adam + all-gather  vs  NCCL all_reduce + Adam

and reports each as a fraction of its roofline: the slower of FLOPs at the
measured bf16 peak and the bytes each rank must move over NVLink at the
measured 770 GB/s per direction. Beside each fused kernel's algorithmic
NVLink bytes it prints the bytes this GPU actually sent and received per
call, from NVML's NVLink throughput counters (read-only queries).
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..ops import native
from ..ops import tp_fused
from ..ops.gemm import EPI_STORE, gemm
from ..parallel import topology
from .kernel_bench import peaks

NVLINK_GBS = 770.0
_NVML_TX, _NVML_RX = 138, 139  # NVML field ids: NVLink data throughput counters (cumulative KiB)


class NvlinkCounters:
    """This GPU's NVLink data bytes sent / received, read from NVML's cumulative
    throughput counters (read-only queries; nothing is configured). Summed over
    the links; ``None`` where the driver offers no such counter."""

    def __init__(self, device_index: int):
        self.h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            props = torch.cuda.get_device_properties(device_index)
            try:  # NVML numbers GPUs by PCI address, CUDA may not
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.links = [ln for ln in range(18) if self._state(ln)]
        except Exception:  # no NVML or no NVLink: the bench still runs
            self.h = None

    def _state(self, link):
        try:
            return self.nvml.nvmlDeviceGetNvLinkState(self.h, link) == 1
        except Exception:
            return False

    def read(self):
        """(tx_bytes, rx_bytes) so far, or None."""
        if self.h is None or not self.links:
            return None
        try:
            tx = rx = 0
            for ln in self.links:
                vals = self.nvml.nvmlDeviceGetFieldValues(self.h, [(_NVML_TX, ln), (_NVML_RX, ln)])
                if any(v.nvmlReturn != 0 for v in vals):
                    return None
                tx += vals[0].value.ullVal
                rx += vals[1].value.ullVal
            return tx * 1024, rx * 1024
        except Exception:
            return None


def nvlink_bytes_per_call(counters, fn, iters=10):
    """NVLink bytes this GPU sent and received per call of ``fn`` (counter
    difference over ``iters`` synchronised calls), or None."""
    torch.cuda.synchronize()
    a = counters.read()
    for _ in range(iters):
        fn()
    torch.cuda.synchronize()
    b = counters.read()
    if a is None or b is None:
        return None
    return {"tx_bytes": (b[0] - a[0]) / iters, "rx_bytes": (b[1] - a[1]) / iters}


def timed(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192, help="B*T per TP group")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--ffn", type=int, default=8192)
    ap.add_argument("--bucket-mb", type=float, default=25.0)
    a = ap.parse_args()
    topology.init_distributed()
    tp = topology.make_tp_context()
    n = tp.world
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(tp.rank)
    tf_peak, _, tag = peaks()
    counters = NvlinkCounters(torch.cuda.current_device())
    M, C, F = a.tokens, a.hidden, a.ffn // n
    rows = M // n
    bf = torch.bfloat16
    out = {"ranks": n, "shape": {"tokens": M, "hidden": C, "ffn_local": F}}

    # ---- AG + GEMM: y[M, F] = AG(x_shard[M/n, C]) W[F, C]^T
    x_shard = torch.randn(rows, C, device=dev, dtype=bf)
    w1 = torch.randn(F, C, device=dev, dtype=bf) * 0.02
    key = 1001
    fused = lambda: tp_fused.ag_gemm(key, "bench.ag", tp, x_shard, a.seq, w1, False, EPI_STORE)  # noqa: E731
    full = torch.empty(M, C, device=dev, dtype=bf)

    def nccl_ag():
        dist.all_gather_into_tensor(full, x_shard, group=tp.group)
        return gemm(full, False, w1, False)

    flops = 2.0 * M * F * C
    nv_bytes = (n - 1) / n * M * C * 2
    roof = max(flops / (tf_peak * 1e12), nv_bytes / (NVLINK_GBS * 1e9)) * 1e3
    t_f, t_n = timed(fused), timed(nccl_ag)
    out["ag_gemm"] = {"fused_ms": t_f, "nccl_gemm_ms": t_n, "roofline_ms": roof, "fraction_of_roofline": roof / t_f,
                      "speedup_vs_nccl": t_n / t_f, "algorithmic_nvlink_bytes": nv_bytes,
                      "nvlink_counters": nvlink_bytes_per_call(counters, fused)}

    # ---- GEMM + RS: y[M/n, C] = RS(h[M, F] W2[C, F]^T)
    h = torch.randn(M, F, device=dev, dtype=bf)
    w2 = torch.randn(C, F, device=dev, dtype=bf) * 0.02
    fused_rs = lambda: tp_fused.gemm_rs(key, "bench.rs", tp, h, a.seq, w2, False)  # noqa: E731
    rs_out = torch.empty(rows, C, device=dev, dtype=bf)

    def nccl_rs():
        y = gemm(h, False, w2, False)
        # sequence sharding: rank r owns tokens [r*T/n, (r+1)*T/n) of each batch row
        yb = y.view(M // a.seq, n, a.seq // n, C).transpose(0, 1).contiguous()
        dist.reduce_scatter_tensor(rs_out, yb.view(n * rows, C), group=tp.group)
        return rs_out

    flops = 2.0 * M * C * F
    nv_bytes = (n - 1) / n * M * C * 2
    roof = max(flops / (tf_peak * 1e12), nv_bytes / (NVLINK_GBS * 1e9)) * 1e3
    t_f, t_n = timed(fused_rs), timed(nccl_rs)
    out["gemm_rs"] = {"fused_ms": t_f, "nccl_gemm_ms": t_n, "roofline_ms": roof, "fraction_of_roofline": roof / t_f,
                      "speedup_vs_nccl": t_n / t_f, "algorithmic_nvlink_bytes": nv_bytes,
                      "nvlink_counters": nvlink_bytes_per_call(counters, fused_rs)}

    # ---- DP bucket: reduce + Adam + all-gather
    from ..optim.fused_dp import FusedDPAdam

    numel = int(a.bucket_mb * 1024 * 1024 / 2)
    p = torch.nn.Parameter(torch.randn(numel, device=dev, dtype=bf) * 0.02)
    mod = torch.nn.Module()
    mod.p = p
    opt = FusedDPAdam(mod, tp, lr=1e-4, bucket_bytes=1 << 40, overlap=False)
    g = torch.randn(numel, device=dev, dtype=bf) * 1e-3

    def fused_dp():
        p.grad = g
        opt.step()

    master = p.detach().float().clone()
    m1, m2 = torch.zeros_like(master), torch.zeros_like(master)
    flat = g.clone()
    step = [0]

    def nccl_dp():
        flat.copy_(g)
        dist.all_reduce(flat, group=tp.group)
        flat.div_(n)
        step[0] += 1
        native.lib().adam_master_step([p.data], [flat], [master], [m1], [m2], 1e-4, 0.9, 0.999, 1e-8, float(step[0]))

    nv_bytes = 2 * (n - 1) / n * numel * 2
    roof = nv_bytes / (NVLINK_GBS * 1e9) * 1e3
    t_f, t_n = timed(fused_dp), timed(nccl_dp)
    out["dp_bucket"] = {"bucket_mb": a.bucket_mb, "fused_ms": t_f, "nccl_adam_ms": t_n, "roofline_ms": roof,
                        "fraction_of_roofline": roof / t_f, "speedup_vs_nccl": t_n / t_f,
                        "algorithmic_nvlink_bytes": nv_bytes, "nvlink_counters": nvlink_bytes_per_call(counters, fused_dp)}
    out["status"] = int(native.lib().read_status(True))
    out["peak"] = f"bf16 {tf_peak} TFLOP/s {tag}; NVLink {NVLINK_GBS} GB/s per direction (measured copy)"
    if tp.rank == 0:
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
