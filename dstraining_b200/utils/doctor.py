"""Check a machine before training on it.

    python -m dstraining_b200.utils.doctor [--json]

Reports, and exits non-zero when a blocking item fails:

* the Python / PyTorch / CUDA / NCCL versions;
* whether the in-tree extension (``dstraining_b200/_C*.so``) imports and
  whether the GPUs are Blackwell data-centre parts (compute capability 10.0,
  the only architecture the kernels are built for) - blocking on a GPU box;
* how many GPUs this process sees and, for every pair, whether one can
  address the other's memory directly (what the NVLink peer-memory kernels
  need; without it TP / DP groups fall back to NCCL);
* per GPU, read through NVML when the ``pynvml`` module is present: active
  NVLink links, current / maximum SM clock and active clock-event reasons
  (read only; nothing is changed);
* the environment settings the framework reads (``CUDA_MODULE_LOADING``,
  ``DST_*``, ``NCCL_*``).

On a machine without GPUs it reports the CPU (gloo) path as usable.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import sys
from typing import Dict, List, Optional

import torch

# clock-event reasons reported, by their pynvml constant names
_REASONS = {
    "GpuIdle": "gpu_idle",
    "ApplicationsClocksSetting": "applications_clocks_setting",
    "SwPowerCap": "sw_power_cap",
    "HwSlowdown": "hw_slowdown",
    "SyncBoost": "sync_boost",
    "SwThermalSlowdown": "sw_thermal_slowdown",
    "HwThermalSlowdown": "hw_thermal_slowdown",
    "HwPowerBrakeSlowdown": "hw_power_brake_slowdown",
    "DisplayClockSetting": "display_clock_setting",
}


def _reason_names(nvml, mask: int) -> List[str]:
    out = []
    for const, name in _REASONS.items():
        bit = getattr(nvml, f"nvmlClocksEventReason{const}", None)
        if bit is None:
            bit = getattr(nvml, f"nvmlClocksThrottleReason{const}", 0)
        if bit and mask & int(bit):
            out.append(name)
    return out


def _nvml_info(n: int, nvml=None) -> Optional[List[Dict]]:
    """Read-only NVML queries per GPU (``None`` without NVML)."""
    if nvml is None:
        try:
            import pynvml as nvml  # nvidia-ml-py
        except ImportError:
            return None
    try:
        nvml.nvmlInit()
    except Exception:  # noqa: BLE001 - no driver: nothing to report
        return None
    out = []
    try:
        for i in range(min(n, nvml.nvmlDeviceGetCount())):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            links = 0
            for link in range(18):
                try:
                    links += int(nvml.nvmlDeviceGetNvLinkState(h, link) == 1)
                except Exception:  # noqa: BLE001 - link index past the device's count
                    break
            reasons = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nvml.nvmlDeviceGetCurrentClocksThrottleReasons
            mask = int(reasons(h))
            out.append({
                "index": i,
                "nvlink_links_active": links,
                "sm_mhz": int(nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)),
                "sm_max_mhz": int(nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM)),
                "clock_event_reasons": _reason_names(nvml, mask),
            })
    finally:
        nvml.nvmlShutdown()
    return out


def collect(nvml=None) -> Dict:
    """Everything :func:`main` prints, as a dict (``problems`` lists the
    blocking failures)."""
    problems: List[str] = []
    notes: List[str] = []
    info: Dict = {
        "python": platform.python_version(),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "nccl": None,
        "gpus": [],
        "peer_access": None,
        "extension": None,
        "env": {k: v for k, v in sorted(os.environ.items())
                if k == "CUDA_MODULE_LOADING" or k.startswith(("DST_", "NCCL_"))},
    }
    try:
        info["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version())
    except Exception:  # noqa: BLE001 - builds without NCCL
        pass
    from ..ops import native

    try:
        native.lib()
        info["extension"] = "loaded"
    except Exception as e:  # noqa: BLE001 - reported
        info["extension"] = f"not loaded: {e}"
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n == 0:
        notes.append("no GPU visible: the CPU (gloo) path runs; native kernels are not used")
    else:
        if info["extension"] != "loaded":
            problems.append("the sm_100a extension does not import (python setup.py build_ext --inplace)")
        for i in range(n):
            p = torch.cuda.get_device_properties(i)
            cc = f"{p.major}.{p.minor}"
            info["gpus"].append({"index": i, "name": p.name, "compute_capability": cc,
                                 "memory_gib": round(p.total_memory / 2**30, 1), "sms": p.multi_processor_count})
            if (p.major, p.minor) != (10, 0):
                problems.append(f"GPU {i} ({p.name}) has compute capability {cc}; the kernels are built for 10.0 "
                                "(sm_100a) only")
        matrix = [[i == j or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)] for i in range(n)]
        info["peer_access"] = matrix
        if n > 1 and not all(all(row) for row in matrix):
            notes.append("some GPU pairs cannot address each other's memory: groups spanning them use NCCL")
        info["nvml"] = _nvml_info(n, nvml)
        for g in info["nvml"] or []:
            bad = [r for r in g["clock_event_reasons"] if r in ("hw_slowdown", "hw_thermal_slowdown",
                                                                   "sw_thermal_slowdown")]
            if bad:
                notes.append(f"GPU {g['index']}: clocks reduced now ({', '.join(bad)})")
    if os.environ.get("CUDA_MODULE_LOADING", "EAGER") != "EAGER":
        notes.append("CUDA_MODULE_LOADING is not EAGER: pipeline ranks can stall on a first kernel launch")
    info["problems"] = problems
    info["notes"] = notes
    return info


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="check this machine for dstraining_b200")
    ap.add_argument("--json", action="store_true", help="print one JSON object")
    a = ap.parse_args(argv)
    info = collect()
    if a.json:
        print(json.dumps(info))
    else:
        for k in ("python", "torch", "cuda_runtime", "nccl", "extension"):
            print(f"{k:14s} {info[k]}")
        for g in info["gpus"]:
            print(f"gpu {g['index']:<10d} {g['name']}  cc {g['compute_capability']}  {g['memory_gib']} GiB  "
                  f"{g['sms']} SMs")
        if info["peer_access"] is not None:
            ok = sum(map(sum, info["peer_access"]))
            print(f"{'peer access':14s} {ok}/{len(info['peer_access']) ** 2} device pairs")
        for g in info.get("nvml") or []:
            print(f"gpu {g['index']:<10d} nvlink links {g['nvlink_links_active']}  sm {g['sm_mhz']}/"
                  f"{g['sm_max_mhz']} MHz  reasons {','.join(g['clock_event_reasons']) or '-'}")
        for k, v in info["env"].items():
            print(f"{'env':14s} {k}={v}")
        for n in info["notes"]:
            print(f"note: {n}")
        for p in info["problems"]:
            print(f"PROBLEM: {p}")
    sys.exit(1 if info["problems"] else 0)


if __name__ == "__main__":
    main()
