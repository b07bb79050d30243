"""bench.py's config table: every layout it offers is a valid process grid
for its model (world size, divisibility rules of the schedules and layers),
and the 8-GPU layouts are the ones BASELINE.json names."""

import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve annotations through it
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_layouts_valid(n):
    bench = _bench()
    for name, cfg in bench.CONFIGS.items():
        lay = cfg.layout(n)
        if lay is None:
            continue
        assert lay["tp"] * lay["pp"] * lay["dp"] == n, (name, n, lay)
        batch = cfg.batch(lay)
        assert batch % cfg.micro == 0, (name, n)
        m = batch // cfg.micro
        assert cfg.heads % lay["tp"] == 0 and (4 * cfg.embd) % lay["tp"] == 0
        assert cfg.block % lay["tp"] == 0
        assert cfg.layers % (lay["pp"] * lay["chunks"]) == 0, (name, n)
        if lay["chunks"] > 1:
            assert m % lay["pp"] == 0, (name, n)  # interleaving needs m % p == 0


def test_baseline_layouts():
    bench = _bench()
    c = bench.CONFIGS
    assert c["c2"].layout(8) == dict(tp=1, pp=1, dp=8, chunks=1) and c["c2"].batch(c["c2"].layout(8)) == 16
    assert c["c3"].layout(8) == dict(tp=8, pp=1, dp=1, chunks=1) and c["c3"].sp and c["c3"].recompute
    assert c["c4"].layout(8) == dict(tp=2, pp=4, dp=1, chunks=2) and c["c4"].batch(c["c4"].layout(8)) == 32
    lay5 = c["c5"].layout(8)
    assert lay5 == dict(tp=2, pp=2, dp=2, chunks=1) and c["c5"].batch(lay5) * lay5["dp"] == 64
    assert bench.parallelism_name(lay5) == "tp2xpp2xdp2"


def test_model_flops():
    bench = _bench()
    c2 = bench.CONFIGS["c2"]
    lay = c2.layout(1)
    n, d, L, V, T = 16 * 1024, 768, 12, 50304, 1024
    want = 3 * n * (24 * d * d * L + 2 * d * V + 2 * T * d * L)
    assert bench.model_flops_per_step(c2, lay) == want
    assert abs(want / 1e12 - 13.08) < 0.05  # GPT-2 small, 16 x 1024 tokens
    assert bench.model_flops_per_step(c2, c2.layout(8)) == 8 * want  # weak scaling: 8 replicas


@pytest.mark.parametrize("impl", ["ours", "reference"])
def test_json_line(impl, monkeypatch, capsys):
    """main() turns one arm's measurements into the one JSON line the driver
    reads (arm faked: no GPU here), with every required key."""
    import json

    bench = _bench()
    for k, v in dict(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0").items():
        monkeypatch.setenv(k, v)
    fake = dict(ms=22.6, e2e_ms=23.0, loss=10.9, launches=(452, 50, [("x", 1)]), h2d=262144, d2h=4, sampler=None,
                status=0, n_params=163_073_280, note=None if impl == "ours" else "stock code path")
    monkeypatch.setattr(bench, "run_ours", lambda *a, **k: fake)
    monkeypatch.setattr(bench, "run_reference", lambda *a, **k: fake)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", impl, "--steps", "5", "--warmup", "3"])
    bench.main()
    line = capsys.readouterr().out.strip().splitlines()[-1]
    out = json.loads(line)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "e2e", "gpu_launches", "impl"):
        assert key in out, key
    assert out["n_gpus"] == 1 and out["steps"] == 5 and out["warmup"] == 3 and out["impl"] == impl
    assert abs(out["value"] - 16 * 1024 / 0.0226) < 1 and out["higher_is_better"] is True
    assert out["config"]["global_batch"] == 16 and out["config"]["seq_len"] == 1024
    assert set(out["e2e"]) >= {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"}
    assert out["gpu_launches"] == (452 * 5 if impl == "ours" else None)
    assert out["model_tflop_per_step"] > 13
