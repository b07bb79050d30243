"""Offline data preparation: local documents -> uint16 train.bin / val.bin
(one end-of-text id per document) that TokenShard reads."""

import json
import os

import numpy as np

from dstraining_b200.utils.data import TokenShard
from dstraining_b200.utils.prepare_data import main, prepare


def test_bytes_tokenizer_roundtrip(tmp_path):
    src = tmp_path / "corpus"
    os.makedirs(src / "sub")
    docs = [f"document number {i}: " + "abc" * (i + 5) for i in range(40)]
    for i, d in enumerate(docs[:30]):
        (src / f"d{i}.txt").write_text(d)
    with open(src / "sub" / "more.jsonl", "w") as f:
        for d in docs[30:]:
            f.write(json.dumps({"text": d}) + "\n")
    out = tmp_path / "data"
    n_train, n_val = prepare([str(src)], str(out), "bytes", val_frac=0.1, seed=1)
    train = np.fromfile(out / "train.bin", dtype=np.uint16)
    val = np.fromfile(out / "val.bin", dtype=np.uint16)
    assert (len(train), len(val)) == (n_train, n_val)
    assert n_train + n_val == sum(len(d.encode()) + 1 for d in docs)
    assert (train == 256).sum() == 36 and (val == 256).sum() == 4  # one end-of-text per document
    # documents decode back intact
    texts = bytes(int(t) for t in train if t != 256).decode() + bytes(int(t) for t in val if t != 256).decode()
    assert sorted(texts.count(f"document number {i}:") for i in range(40)) == [1] * 40
    x, y = TokenShard(str(out / "train.bin"), block_size=16, batch_size=4, seed=0).get_batch(3)
    assert x.shape == (4, 16) and bool((x[:, 1:] == y[:, :-1]).all())


def test_cli_doc_separator(tmp_path):
    (tmp_path / "a.txt").write_text("one\n\ntwo\n\nthree")
    main(["--input", str(tmp_path / "a.txt"), "--out", str(tmp_path / "o"), "--val-frac", "0", "--doc-sep", "\n\n"])
    train = np.fromfile(tmp_path / "o" / "train.bin", dtype=np.uint16)
    assert (train == 256).sum() == 3 and os.path.getsize(tmp_path / "o" / "val.bin") == 0


def test_tokenizer_json(tmp_path):
    """A tokenizer.json (built here offline: word-level, with an end-of-text
    token) through the multi-process path."""
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace

    vocab = {"<|endoftext|>": 0, "[UNK]": 1, "hello": 2, "world": 3, "again": 4}
    tok = Tokenizer(WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = Whitespace()
    tok.save(str(tmp_path / "tokenizer.json"))
    with open(tmp_path / "c.jsonl", "w") as f:
        for _ in range(8):
            f.write(json.dumps({"text": "hello world again hello"}) + "\n")
    prepare([str(tmp_path / "c.jsonl")], str(tmp_path / "o"), str(tmp_path / "tokenizer.json"),
            val_frac=0.25, num_proc=2)
    train = np.fromfile(tmp_path / "o" / "train.bin", dtype=np.uint16)
    assert train.tolist() == [2, 3, 4, 2, 0] * 6


def test_train_on_prepared_data(tmp_path):
    """prepare_data -> train.py --data train.bin --eval-data val.bin on 2 gloo
    ranks (data parallel); the held-out loss is logged."""
    from dstraining_b200.utils.launch import launch

    src = tmp_path / "corpus"
    os.makedirs(src)
    for i in range(60):
        (src / f"d{i}.txt").write_text(("the quick brown fox jumps over the lazy dog %d. " % i) * 20)
    prepare([str(src)], str(tmp_path / "data"), "bytes", val_frac=0.1, seed=0)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sink = tmp_path / "m.jsonl"
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    argv = [os.path.join(root, "train.py"), "--dp", "2", "--layers", "1", "--heads", "2", "--embd", "32",
            "--block", "64", "--vocab", "257", "--batch", "4", "--steps", "4", "--device", "cpu",
            "--data", str(tmp_path / "data" / "train.bin"), "--eval-data", str(tmp_path / "data" / "val.bin"),
            "--eval-every", "2", "--jsonl", str(sink)]
    assert launch(2, argv, timeout=300, env=env) == 0
    recs = [json.loads(ln) for ln in sink.read_text().splitlines()]
    evals = [r["eval_loss"] for r in recs if "eval_loss" in r]
    assert len(evals) == 2 and all(np.isfinite(evals))
