"""Sampling from a trained model.

    python -m dstraining_b200.utils.generate --ckpt ckpt/ --text "hello" --tokenizer bytes \
        --max-new-tokens 64 [--temperature 0.8 --top-k 40 --seed 0]

``generate(model, idx, ...)`` extends ``idx`` [B, T] token by token with the
full-context forward pass (no KV cache): the last ``block_size`` tokens are
the context, right-padded to a multiple of ``pad_to`` so the native causal
attention kernels (which take sequence lengths in multiples of 64 / 128) can
run it - under causal attention the padding never influences the positions
before it. ``temperature == 0`` is greedy decoding. Works for ``GPT`` at any
tensor-parallel degree (every TP rank must call it with the same inputs and
generator state); pipeline stages are not supported. The CLI loads a sharded
checkpoint (any layout) into a single-process model. The reference has no
sampling code.
"""

from __future__ import annotations

import argparse
import json
import os
from typing import Optional

import torch

from ..models.gpt import GPT, GPTConfig
from ..parallel.topology import SINGLE


@torch.no_grad()
def generate(model: GPT, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
             top_k: Optional[int] = None, generator: Optional[torch.Generator] = None, pad_to: int = 128) -> torch.Tensor:
    cfg = model.config
    was_training = model.training
    model.eval()
    try:
        for _ in range(max_new_tokens):
            ctx = idx[:, -cfg.block_size:]
            n = ctx.shape[1]
            padded = min(cfg.block_size, -(-n // pad_to) * pad_to) if pad_to > 1 else n
            if padded > n:
                ctx = torch.cat([ctx, ctx.new_zeros(ctx.shape[0], padded - n)], dim=1)
            logits, _ = model(ctx)
            logits = logits[:, n - 1, : cfg.vocab_size].float()
            if temperature <= 0:
                nxt = logits.argmax(dim=-1, keepdim=True)
            else:
                logits = logits / temperature
                if top_k is not None and top_k < logits.shape[-1]:
                    kth = torch.topk(logits, top_k, dim=-1).values[:, -1:]
                    logits = logits.masked_fill(logits < kth, float("-inf"))
                probs = torch.softmax(logits, dim=-1)
                nxt = torch.multinomial(probs.cpu(), 1, generator=generator).to(idx.device)
            idx = torch.cat([idx, nxt.to(idx.dtype)], dim=1)
    finally:
        model.train(was_training)
    return idx


def load_model(ckpt: str, device: str = "cpu", dtype: torch.dtype = torch.float32) -> GPT:
    """A single-process GPT holding the weights of a sharded checkpoint (a step
    directory, or a root whose latest complete checkpoint is used)."""
    from . import checkpoint

    path = ckpt if os.path.exists(os.path.join(ckpt, "manifest.json")) else checkpoint.latest(ckpt)
    if path is None:
        raise FileNotFoundError(f"no complete checkpoint under {ckpt}")
    with open(os.path.join(path, "manifest.json")) as f:
        conf = json.load(f)["config"]
    fields = set(GPTConfig.__dataclass_fields__)
    cfg = GPTConfig(**{k: v for k, v in conf.items() if k in fields and k != "sequence_parallel"})
    model = GPT(cfg, SINGLE, seed=0)
    checkpoint.load(path, model, None, SINGLE)
    return model.to(device).to(dtype)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="sample from a trained checkpoint")
    ap.add_argument("--ckpt", required=True)
    ap.add_argument("--text", default=None, help="prompt text (needs --tokenizer)")
    ap.add_argument("--tokens", default=None, help="prompt as comma-separated token ids")
    ap.add_argument("--tokenizer", default="bytes", help="'bytes' or a tokenizer.json path")
    ap.add_argument("--max-new-tokens", type=int, default=64)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--top-k", type=int, default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dtype = torch.bfloat16 if a.device.startswith("cuda") else torch.float32
    model = load_model(a.ckpt, a.device, dtype)
    if a.tokens:
        ids = [int(t) for t in a.tokens.split(",")]
        decode = None
    else:
        from .prepare_data import make_tokenizer

        tok = make_tokenizer(a.tokenizer)
        ids = tok.encode(a.text or "")
        if not ids:
            ids = [tok.eot]
        decode = (lambda out: bytes(t for t in out if t < 256).decode("utf-8", "replace")) if a.tokenizer == "bytes" \
            else (lambda out: tok.tok.decode(out))
    idx = torch.tensor([ids], dtype=torch.long, device=a.device)
    g = torch.Generator().manual_seed(a.seed)
    out = generate(model, idx, a.max_new_tokens, a.temperature, a.top_k, g)[0].tolist()
    print(decode(out) if decode else ",".join(map(str, out)))


if __name__ == "__main__":
    main()
