"""Layout planner: parameter counts per rank match the models actually built
(every TP rank and pipeline stage), and invalid or slow layouts are reported."""

import pytest

from dstraining_b200.models.gpt import GPT, GPTConfig, GPTStage
from dstraining_b200.parallel.topology import PPContext, TPContext
from dstraining_b200.trainer import parse_args
from dstraining_b200.utils.plan import main, plan, stage_params

BASE = ["--layers", "4", "--heads", "4", "--embd", "64", "--block", "128", "--vocab", "300"]


@pytest.mark.parametrize("tp,pp", [(1, 1), (2, 1), (4, 1), (2, 2), (1, 4)])
def test_param_counts_match_models(tp, pp):
    args = parse_args([*BASE, "--tp", str(tp), "--pp", str(pp)])
    cfg = GPTConfig(vocab_size=300, block_size=128, n_layer=4, n_head=4, n_embd=64)
    for s in range(pp):
        for r in range(tp):
            tpc = TPContext(group=None, rank=r, world=tp)
            if pp == 1:
                m = GPT(cfg, tpc, seed=1)
            else:
                ppc = PPContext(rank=s, world=pp, prev_rank=None, next_rank=None, ring_prev_rank=None,
                                ring_next_rank=None)
                m = GPTStage(cfg, tpc, ppc, seed=1)
            assert sum(p.numel() for p in m.parameters()) == stage_params(args, s, tp), (tp, pp, s, r)


def test_reports_invalid_and_slow_layouts(capsys):
    bad = plan(parse_args([*BASE, "--tp", "3", "--pp", "3"]))
    assert not bad["valid"] and len(bad["errors"]) >= 2
    slow = plan(parse_args(["--layers", "4", "--heads", "4", "--embd", "256", "--block", "192", "--vocab", "300",
                            "--tp", "2", "--sp", "--bf16"]))
    assert slow["valid"] and any("fused TP" in w for w in slow["fast_path_warnings"])
    assert any("zero-pads it to 256" in w for w in slow["fast_path_warnings"])
    good = plan(parse_args(["--layers", "24", "--heads", "16", "--embd", "2048", "--block", "2048", "--vocab",
                            "50304", "--tp", "2", "--pp", "2", "--dp", "2", "--sp", "--bf16", "--vp", "--batch", "32",
                            "--micro", "2"]))
    assert good["valid"] and not good["fast_path_warnings"] and good["micro_batches"] == 16
    assert good["optimizer"].startswith("fused")
    with pytest.raises(SystemExit) as e:
        main([*BASE, "--tp", "2"])
    assert e.value.code == 0 and '"valid": true' in capsys.readouterr().out


def test_gpt2_preset():
    # GPT-2 124M shape with an untied head over the padded vocabulary: 163,073,280 parameters
    out = plan(parse_args(["--gpt2", "--bf16", "--vp", "--batch", "16"]))
    assert out["valid"] and out["per_stage"][0]["params"] == 50257 * 768 + 1024 * 768 + 12 * (12 * 768 * 768 + 13 * 768) \
        + 2 * 768 + 50304 * 768
    assert out["tokens_per_step"] == 16 * 1024


def test_plain_tp_runs_fused_without_warning():
    """Plain TP (no SP) keeps every TP collective on the fused NVLink kernels,
    the MLP included, so the planner has nothing to warn about."""
    out = plan(parse_args(["--layers", "4", "--heads", "4", "--embd", "256", "--block", "256", "--vocab", "300",
                           "--tp", "2", "--bf16"]))
    assert out["valid"] and not any("without --sp" in w for w in out["fast_path_warnings"])
