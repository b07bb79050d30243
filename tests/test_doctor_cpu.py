"""Machine check: on a machine without GPUs it reports the CPU path as usable
and exits 0; NVML answers (a fake NVML here: read-only queries) are decoded
into link counts, clocks and clock-event reason names."""

import json
import types

import pytest

from dstraining_b200.utils import doctor


def test_cpu_machine(capsys):
    with pytest.raises(SystemExit) as e:
        doctor.main(["--json"])
    assert e.value.code == 0
    info = json.loads(capsys.readouterr().out)
    assert info["problems"] == [] and info["torch"] and info["extension"]


def test_fake_nvml():
    calls = []

    class H:
        pass

    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=1,
        nvmlClocksEventReasonSwPowerCap=0x4,
        nvmlClocksEventReasonHwSlowdown=0x8,
        nvmlClocksEventReasonGpuIdle=0x1,
        nvmlInit=lambda: calls.append("init"),
        nvmlShutdown=lambda: calls.append("shutdown"),
        nvmlDeviceGetCount=lambda: 2,
        nvmlDeviceGetHandleByIndex=lambda i: H(),
        nvmlDeviceGetNvLinkState=lambda h, link: 1 if link < 18 else 0,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4 | 0x8,
        nvmlDeviceGetClockInfo=lambda h, kind: 1335,
        nvmlDeviceGetMaxClockInfo=lambda h, kind: 1965,
    )
    out = doctor._nvml_info(2, fake)
    assert calls == ["init", "shutdown"] and len(out) == 2
    assert out[0]["nvlink_links_active"] == 18 and out[0]["sm_mhz"] == 1335 and out[0]["sm_max_mhz"] == 1965
    assert out[0]["clock_event_reasons"] == ["sw_power_cap", "hw_slowdown"]
