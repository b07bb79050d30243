"""Export to the Hugging Face GPT-2 layout: ``transformers.GPT2LMHeadModel``
loaded from the exported files gives this model's logits (real vocabulary)
and loss; the CLI exports a sharded tp=2 checkpoint."""

import os

import torch

from dstraining_b200.models.gpt import GPT, GPTConfig
from dstraining_b200.parallel.topology import SINGLE
from dstraining_b200.utils.export_hf import export, main
from dstraining_b200.utils.launch import launch


def test_logits_match_transformers(tmp_path):
    from transformers import GPT2LMHeadModel

    cfg = GPTConfig(vocab_size=300, block_size=64, n_layer=2, n_head=4, n_embd=64)
    m = GPT(cfg, SINGLE, seed=11).eval()
    export(m, str(tmp_path / "hf"))
    hf = GPT2LMHeadModel.from_pretrained(str(tmp_path / "hf")).eval()
    idx = torch.randint(0, 300, (2, 48), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        ours, _ = m(idx)
        theirs = hf(idx).logits
        _, loss = m(idx, idx)
        hf_loss = torch.nn.functional.cross_entropy(theirs.reshape(-1, 300), idx.reshape(-1))
    torch.testing.assert_close(theirs, ours[..., :300], atol=2e-5, rtol=1e-5)
    torch.testing.assert_close(hf_loss, loss, atol=1e-5, rtol=1e-5)


def test_cli_from_tp2_checkpoint(tmp_path):
    from transformers import GPT2LMHeadModel

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    argv = [os.path.join(root, "train.py"), "--tp", "2", "--layers", "1", "--heads", "2", "--embd", "32",
            "--block", "32", "--vocab", "257", "--batch", "2", "--steps", "2", "--device", "cpu",
            "--ckpt-dir", str(tmp_path / "ck")]
    assert launch(2, argv, timeout=300, env=env) == 0
    main(["--ckpt", str(tmp_path / "ck"), "--out", str(tmp_path / "hf"), "--dtype", "bfloat16"])
    hf = GPT2LMHeadModel.from_pretrained(str(tmp_path / "hf"))
    assert hf.config.vocab_size == 257 and hf.lm_head.weight.shape == (257, 32)
    assert hf.lm_head.weight.data_ptr() != hf.transformer.wte.weight.data_ptr()


def test_import_transformers_model(tmp_path):
    """A GPT-2 saved by transformers (tied head) imports with the same logits,
    and fine-tuning starts from it at another layout (tp=2, resharded)."""
    from transformers import GPT2Config, GPT2LMHeadModel

    from dstraining_b200.utils import checkpoint
    from dstraining_b200.utils.export_hf import import_hf

    torch.manual_seed(0)
    hf = GPT2LMHeadModel(GPT2Config(vocab_size=200, n_positions=32, n_embd=32, n_layer=2, n_head=2,
                                    resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0)).eval()
    hf.save_pretrained(str(tmp_path / "hf"))
    m = import_hf(str(tmp_path / "hf")).eval()
    idx = torch.randint(0, 200, (2, 32), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        torch.testing.assert_close(m(idx)[0][..., :200], hf(idx).logits, atol=2e-5, rtol=1e-5)
    main(["--import-hf", str(tmp_path / "hf"), "--ckpt", str(tmp_path / "ck")])
    assert checkpoint.latest(str(tmp_path / "ck")).endswith("step_00000000")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    argv = [os.path.join(root, "train.py"), "--tp", "2", "--layers", "2", "--heads", "2", "--embd", "32",
            "--block", "32", "--vocab", "200", "--batch", "2", "--steps", "2", "--device", "cpu",
            "--ckpt-dir", str(tmp_path / "ck"), "--resume"]
    assert launch(2, argv, timeout=300, env=env) == 0
    assert checkpoint.latest(str(tmp_path / "ck")).endswith("step_00000002")
