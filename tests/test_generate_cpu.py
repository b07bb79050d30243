"""Sampling: right-padding the context (for the native attention kernels)
does not change greedy outputs; the KV-cache decoder gives the full-context
forward pass's logits and tokens (also once the window slides); the CLI
samples from a sharded checkpoint written at tp=2."""

import os

import torch

from dstraining_b200.models.gpt import GPT, GPTConfig
from dstraining_b200.parallel.topology import SINGLE
from dstraining_b200.utils.generate import KVCache, generate, main
from dstraining_b200.utils.launch import launch


def test_padding_does_not_change_greedy_output():
    cfg = GPTConfig(vocab_size=300, block_size=64, n_layer=2, n_head=4, n_embd=64)
    m = GPT(cfg, SINGLE, seed=5)
    idx = torch.randint(0, 300, (2, 7), generator=torch.Generator().manual_seed(1))
    a = generate(m, idx, 70, temperature=0.0, pad_to=1, use_cache=False)  # crosses block_size: the window slides
    b = generate(m, idx, 70, temperature=0.0, pad_to=32, use_cache=False)
    assert a.shape == (2, 77) and torch.equal(a, b)
    g1, g2 = torch.Generator().manual_seed(3), torch.Generator().manual_seed(3)
    s1 = generate(m, idx, 10, temperature=0.9, top_k=20, generator=g1)
    s2 = generate(m, idx, 10, temperature=0.9, top_k=20, generator=g2)
    assert torch.equal(s1, s2)  # seeded sampling is reproducible


def test_cli_from_tp2_checkpoint(tmp_path, capsys):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    argv = [os.path.join(root, "train.py"), "--tp", "2", "--layers", "1", "--heads", "2", "--embd", "32",
            "--block", "32", "--vocab", "257", "--batch", "2", "--steps", "2", "--device", "cpu",
            "--ckpt-dir", str(tmp_path / "ck")]
    assert launch(2, argv, timeout=300, env=env) == 0
    main(["--ckpt", str(tmp_path / "ck"), "--text", "hi", "--max-new-tokens", "6", "--temperature", "0",
          "--device", "cpu"])
    out = capsys.readouterr().out.rstrip("\n")
    assert out.startswith("hi")
    main(["--ckpt", str(tmp_path / "ck"), "--tokens", "104,105", "--max-new-tokens", "6", "--temperature", "0",
          "--device", "cpu"])
    assert len(capsys.readouterr().out.strip().split(",")) == 8


def test_kv_cache_matches_full_context():
    cfg = GPTConfig(vocab_size=300, block_size=64, n_layer=2, n_head=4, n_embd=64)
    m = GPT(cfg, SINGLE, seed=7).eval()
    seq = torch.randint(0, 300, (3, 40), generator=torch.Generator().manual_seed(2))
    cache = KVCache(m, 3)
    with torch.no_grad():
        got = [cache.forward(seq[:, :9])]  # the prompt, then one token at a time
        got += [cache.forward(seq[:, t : t + 1]) for t in range(9, 40)]
        full, _ = m(seq)
    want = full[:, 8:, :300]
    torch.testing.assert_close(torch.stack(got, dim=1), want, atol=2e-5, rtol=1e-5)
    idx = seq[:, :5]
    a = generate(m, idx, 80, temperature=0.0, use_cache=True)  # past block_size: full-window steps
    b = generate(m, idx, 80, temperature=0.0, use_cache=False, pad_to=1)
    assert a.shape == (3, 85) and torch.equal(a, b)


def test_top_p_keeps_the_nucleus():
    from dstraining_b200.utils.generate import _sample

    logits = torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]]))
    g = torch.Generator().manual_seed(0)
    draws = {int(_sample(logits, 1.0, None, g, top_p=0.7)) for _ in range(200)}
    assert draws == {0, 1}  # 0.5 + 0.3 covers 0.7; tokens 2 and 3 are cut
    draws = {int(_sample(logits, 1.0, None, g, top_p=0.1)) for _ in range(50)}
    assert draws == {0}  # always at least the most probable token


def test_kv_cache_tensor_parallel():
    """tp=2 (gloo): the cached decoder gives the tp=1 logits and tokens."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    assert launch(2, [os.path.join(root, "tests", "suites", "kv_tp_suite.py"), "--device", "cpu"], timeout=300,
                  env=env) == 0
