"""Timeline tracing: NVTX ranges (``DST_NVTX=1``) and ``torch.profiler``
windows (``train.py --profile-dir``: a Chrome trace and a per-kernel
device-time table per rank).

``nvtx_range(name)`` is a context manager that pushes an NVTX range around
its body when ``DST_NVTX`` is set and CUDA is available, and marks the same
range in a running :class:`StepProfiler` window; otherwise it does nothing
(no cost on the normal path). The trainer marks its phases
(``forward_backward``, ``dp_reduce``, ``finalize_grads``, ``optimizer``) and
the models mark each block, so a timeline shows where a step's time goes.
:class:`StepProfiler` records a window of steps with ``torch.profiler`` (host
ops and, on CUDA, every kernel) and writes one Chrome trace per rank. The
reference has no tracing (its only timing is a cumulative wall-clock average
in ``train.py:123-152``).
"""

from __future__ import annotations

import contextlib
import os

import torch


_PROFILING = False  # a StepProfiler window is recording


def enabled() -> bool:
    return (os.environ.get("DST_NVTX", "0") not in ("", "0") and torch.cuda.is_available()) or _PROFILING


@contextlib.contextmanager
def nvtx_range(name: str):
    if not enabled():
        yield
        return
    nvtx = os.environ.get("DST_NVTX", "0") not in ("", "0") and torch.cuda.is_available()
    if nvtx:
        torch.cuda.nvtx.range_push(name)
    try:
        if _PROFILING:
            with torch.profiler.record_function(name):
                yield
        else:
            yield
    finally:
        if nvtx:
            torch.cuda.nvtx.range_pop()


class StepProfiler:
    """Records steps ``[start, start + count)`` with ``torch.profiler`` and
    writes ``<out_dir>/trace_rank<R>.json`` (Chrome trace format; open it in
    Perfetto or chrome://tracing). Call :meth:`before` and :meth:`after`
    around every step."""

    def __init__(self, out_dir: str, start: int, count: int, rank: int, cuda: bool):
        self.out_dir, self.start, self.end, self.rank, self.cuda = out_dir, start, start + count, rank, cuda
        self.prof = None
        self.path = None

    def before(self, step: int) -> None:
        global _PROFILING
        if step == self.start:
            acts = [torch.profiler.ProfilerActivity.CPU]
            if self.cuda:
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self.prof = torch.profiler.profile(activities=acts)
            self.prof.__enter__()
            _PROFILING = True

    def after(self, step: int) -> None:
        if self.prof is not None and step == self.end - 1:
            self.close()

    def close(self) -> None:
        """Stop a window still open (a run shorter than the window) and write it."""
        global _PROFILING
        if self.prof is None:
            return
        if self.cuda:
            torch.cuda.synchronize()
        self.prof.__exit__(None, None, None)
        _PROFILING = False
        os.makedirs(self.out_dir, exist_ok=True)
        self.path = os.path.join(self.out_dir, f"trace_rank{self.rank}.json")
        self.prof.export_chrome_trace(self.path)
        if self.cuda:
            with open(os.path.join(self.out_dir, f"kernels_rank{self.rank}.txt"), "w") as f:
                f.write(kernel_summary(self.prof, self.end - self.start))
        self.prof = None


def busy_time(spans) -> float:
    """Length of the union of ``(start, end)`` intervals (overlapping kernels
    on several streams count once)."""
    spans = sorted(spans)
    busy, cur_s, cur_e = 0.0, spans[0][0], spans[0][1]
    for s0, e0 in spans[1:]:
        if s0 > cur_e:
            busy += cur_e - cur_s
            cur_s, cur_e = s0, e0
        else:
            cur_e = max(cur_e, e0)
    return busy + (cur_e - cur_s)


def kernel_summary(prof, steps: int = 1) -> str:
    """Device time per kernel name over a recorded window: calls and
    microseconds per step, share of the summed kernel time, and the device
    busy fraction (union of kernel intervals over the span from the first
    kernel's start to the last one's end; below 1 means the GPU waited for the
    host or for other GPUs)."""
    rows, spans = {}, []
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA or getattr(ev, "is_user_annotation", False):
            continue  # device-side copies of the host's named ranges are not kernels
        name = ev.name
        if name.startswith("Memcpy") or name.startswith("Memset"):
            kind = name.split()[0]
        else:
            kind = name
        dur = ev.time_range.end - ev.time_range.start  # microseconds
        r = rows.setdefault(kind, [0, 0.0])
        r[0] += 1
        r[1] += dur
        spans.append((ev.time_range.start, ev.time_range.end))
    if not spans:
        return "no device activity recorded\n"
    busy = busy_time(spans)
    wall = max(e for _, e in spans) - min(s for s, _ in spans)
    total = sum(v[1] for v in rows.values())
    out = [f"window: {steps} step(s); span {wall / steps:.1f} us/step; device busy {busy / steps:.1f} us/step "
           f"({busy / wall:.1%} of the span); summed kernel time {total / steps:.1f} us/step",
           f"{'us/step':>10s} {'share':>7s} {'calls/step':>10s}  kernel"]
    for kind, (n, t) in sorted(rows.items(), key=lambda kv: -kv[1][1]):
        out.append(f"{t / steps:10.1f} {t / total:7.1%} {n / steps:10.1f}  {kind[:150]}")
    return "\n".join(out) + "\n"
