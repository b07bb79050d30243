"""Tokenise local text into flat uint16 token files for :class:`TokenShard`.

    python -m dstraining_b200.utils.prepare_data --input corpus/ --out data \
        --tokenizer path/to/tokenizer.json [--val-frac 0.0005] [--num-proc 8]

Writes ``<out>/train.bin`` and ``<out>/val.bin``: token ids as raw uint16,
one end-of-text token after every document - the same file format the
reference's ``scripts/prepare_openwebtext.py:15-50`` produces (it downloads
OpenWebText and uses the GPT-2 BPE, which needs network access; this one
reads local files, so it works offline).

Documents: every line of a ``.jsonl`` file (its ``"text"`` field), or every
``.txt`` file (split further on ``--doc-sep`` if given). Directories are
searched recursively. Documents are shuffled with ``--seed`` and a
``--val-frac`` share goes to ``val.bin``, as in the reference (0.0005,
seed 2357).

Tokenizers: ``--tokenizer bytes`` (UTF-8 bytes, ids 0-255, end-of-text 256),
or a Hugging Face ``tokenizer.json`` file (its ``--eot`` token, default
``<|endoftext|>``). Ids must fit in uint16.
"""

from __future__ import annotations

import argparse
import json
import os
import random
from multiprocessing import get_context
from typing import Iterable, List, Optional, Sequence, Tuple

import numpy as np

_TOK = None  # per-worker tokenizer


def iter_documents(paths: Sequence[str], doc_sep: Optional[str] = None) -> Iterable[str]:
    files: List[str] = []
    for p in paths:
        if os.path.isdir(p):
            for root, _, names in os.walk(p):
                files.extend(os.path.join(root, n) for n in names if n.endswith((".txt", ".jsonl")))
        else:
            files.append(p)
    for f in sorted(files):
        with open(f, encoding="utf-8") as fh:
            if f.endswith(".jsonl"):
                for line in fh:
                    line = line.strip()
                    if line:
                        yield json.loads(line)["text"]
            else:
                text = fh.read()
                parts = text.split(doc_sep) if doc_sep else [text]
                for part in parts:
                    if part.strip():
                        yield part


class _Bytes:
    eot = 256

    def encode(self, text: str) -> List[int]:
        return list(text.encode("utf-8"))


class _HF:
    def __init__(self, path: str, eot: str):
        from tokenizers import Tokenizer

        self.tok = Tokenizer.from_file(path)
        eid = self.tok.token_to_id(eot)
        if eid is None:
            raise ValueError(f"tokenizer {path} has no token {eot!r}")
        self.eot = eid

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text, add_special_tokens=False).ids


def make_tokenizer(spec: str, eot: str = "<|endoftext|>"):
    return _Bytes() if spec == "bytes" else _HF(spec, eot)


def _init_worker(spec: str, eot: str) -> None:
    global _TOK
    _TOK = make_tokenizer(spec, eot)


def _encode(text: str) -> np.ndarray:
    ids = _TOK.encode(text)
    ids.append(_TOK.eot)
    arr = np.asarray(ids, dtype=np.int64)
    if arr.size and (arr.max() > np.iinfo(np.uint16).max or arr.min() < 0):
        raise ValueError("token id does not fit in uint16")
    return arr.astype(np.uint16)


def write_bin(path: str, chunks: Sequence[np.ndarray]) -> int:
    total = int(sum(c.size for c in chunks))
    arr = np.memmap(path, dtype=np.uint16, mode="w+", shape=(max(total, 1),))
    pos = 0
    for c in chunks:
        arr[pos : pos + c.size] = c
        pos += c.size
    arr.flush()
    del arr
    if total == 0:
        open(path, "wb").close()
    return total


def prepare(inputs: Sequence[str], out: str, tokenizer: str = "bytes", eot: str = "<|endoftext|>",
            val_frac: float = 0.0005, seed: int = 2357, num_proc: int = 1,
            doc_sep: Optional[str] = None) -> Tuple[int, int]:
    """Tokenise and write ``train.bin`` / ``val.bin``; returns their token counts."""
    docs = list(iter_documents(inputs, doc_sep))
    if not docs:
        raise ValueError("no documents found")
    random.Random(seed).shuffle(docs)
    n_val = int(round(len(docs) * val_frac))
    if val_frac > 0 and len(docs) > 1:
        n_val = max(1, n_val)
    val_docs, train_docs = docs[:n_val], docs[n_val:]
    os.makedirs(out, exist_ok=True)
    counts = []
    for name, part in (("train", train_docs), ("val", val_docs)):
        if num_proc > 1:
            # spawned workers: forking a process that already runs threads (torch) is unsafe
            with get_context("spawn").Pool(num_proc, initializer=_init_worker, initargs=(tokenizer, eot)) as pool:
                chunks = pool.map(_encode, part, chunksize=64)
        else:
            _init_worker(tokenizer, eot)
            chunks = [_encode(t) for t in part]
        n = write_bin(os.path.join(out, f"{name}.bin"), chunks)
        counts.append(n)
        print(f"{os.path.join(out, name + '.bin')}: {n:,} tokens from {len(part):,} documents", flush=True)
    return counts[0], counts[1]


def main(argv: Optional[Sequence[str]] = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--input", nargs="+", required=True, help="text / jsonl files or directories")
    ap.add_argument("--out", default="data")
    ap.add_argument("--tokenizer", default="bytes", help="'bytes' or a tokenizer.json path")
    ap.add_argument("--eot", default="<|endoftext|>", help="end-of-text token of a tokenizer.json")
    ap.add_argument("--val-frac", type=float, default=0.0005)
    ap.add_argument("--seed", type=int, default=2357)
    ap.add_argument("--num-proc", type=int, default=1)
    ap.add_argument("--doc-sep", default=None, help="split .txt files into documents on this string")
    a = ap.parse_args(argv)
    prepare(a.input, a.out, a.tokenizer, a.eot, a.val_frac, a.seed, a.num_proc, a.doc_sep)


if __name__ == "__main__":
    main()
