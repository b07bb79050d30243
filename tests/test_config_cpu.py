"""train.py --config: YAML flag defaults, command line wins, unknown keys rejected."""

import pytest

from dstraining_b200.trainer import parse_args


def test_yaml_defaults_and_precedence(tmp_path):
    cfg = tmp_path / "c.yaml"
    cfg.write_text("tp: 2\nsp: true\nlearning-rate-typo: 1\n")
    with pytest.raises(ValueError, match="unknown flag"):
        parse_args(["--config", str(cfg)])
    cfg.write_text("tp: 2\nsp: true\nlr: 0.01\nbucket-mb: 8\n")
    a = parse_args(["--config", str(cfg), "--lr", "0.002"])
    assert a.tp == 2 and a.sp is True and a.bucket_mb == 8 and a.lr == 0.002
    b = parse_args([])
    assert b.tp == 1 and b.config is None
