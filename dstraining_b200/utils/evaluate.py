"""Held-out loss and perplexity of a checkpoint on token files.

    python -m dstraining_b200.utils.evaluate --ckpt ckpt/ --data data/val.bin [--max-tokens 1000000]

Loads the checkpoint (any training layout) into a single-process model and
runs it over consecutive, non-overlapping ``block_size`` windows of the
token files (``--data`` as in ``train.py``: a file, a directory, a glob or a
list), in batches of ``--batch`` windows; every window predicts its next
``block_size`` tokens. Prints one JSON line: tokens scored, mean loss
(nats per token) and perplexity. Unlike ``train.py --eval-every``, which
samples random windows, this reads the files in order, so the result is a
fixed number for a given checkpoint and data.
"""

from __future__ import annotations

import argparse
import json
import math
from typing import Dict, Optional

import numpy as np
import torch

from .data import token_files


@torch.no_grad()
def evaluate(model, data: str, batch: int = 8, max_tokens: Optional[int] = None, device: str = "cpu") -> Dict:
    """Mean next-token loss of ``model`` over consecutive windows of ``data``."""
    cfg = model.config
    T = cfg.block_size
    was_training = model.training
    model.eval()
    total, count = 0.0, 0
    try:
        windows = []
        for f in token_files(data):
            arr = np.memmap(f, dtype=np.uint16, mode="r")
            for s in range(0, len(arr) - T - 1 + 1, T):
                windows.append((arr, s))
        if max_tokens is not None:
            windows = windows[: max(1, max_tokens // T)]
        for i in range(0, len(windows), batch):
            part = windows[i : i + batch]
            rows = torch.from_numpy(np.stack([np.asarray(a[s : s + T + 1]) for a, s in part]).astype(np.int64))
            x, y = rows[:, :-1].to(device), rows[:, 1:].to(device)
            _, loss = model(x, y)
            n = y.numel()
            total += float(loss.float()) * n
            count += n
    finally:
        model.train(was_training)
    if count == 0:
        raise ValueError(f"{data}: no file holds a full window of {T + 1} tokens")
    mean = total / count
    return {"tokens": count, "loss": mean, "perplexity": math.exp(mean)}


def main(argv=None) -> None:
    from .generate import load_model

    ap = argparse.ArgumentParser(description="held-out loss and perplexity of a checkpoint")
    ap.add_argument("--ckpt", required=True)
    ap.add_argument("--data", required=True, help="token file(s): file, directory, glob or comma-separated list")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--max-tokens", type=int, default=None)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dtype = torch.bfloat16 if a.device.startswith("cuda") else torch.float32
    model = load_model(a.ckpt, a.device, dtype)
    print(json.dumps({"ckpt": a.ckpt, "data": a.data, **evaluate(model, a.data, a.batch, a.max_tokens, a.device)}))


if __name__ == "__main__":
    main()
