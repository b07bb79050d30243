"""Sampling from a trained model.

    python -m dstraining_b200.utils.generate --ckpt ckpt/ --text "hello" --tokenizer bytes \
        --max-new-tokens 64 [--temperature 0.8 --top-k 40 --seed 0]

``generate(model, idx, ...)`` extends ``idx`` [B, T] token by token.
``temperature == 0`` is greedy decoding; otherwise tokens are sampled,
optionally from the ``top_k`` most probable and / or the nucleus of
probability ``top_p``.

* With ``use_cache=True`` (the default) the prompt is run once and every
  later token costs one row per layer: its key and value are appended to a
  per-layer cache and its query attends over the cache (under tensor
  parallelism each rank caches its own heads; every rank of the group must
  call it with the same inputs and generator state).
  Positions are learned and absolute, so once the sequence outgrows
  ``block_size`` the window slides and every step re-runs the whole window,
  exactly as without a cache. Runs on the model's own parameters with
  PyTorch ops (fp32 on CPU, the model's dtype on CUDA).
* Otherwise every step runs the model's full-context forward pass on the
  last ``block_size`` tokens, right-padded to a multiple of ``pad_to`` (the
  native causal attention kernels' 128-row tiles, so the sequence-parallel
  and fused tensor-parallel layers see whole tiles too) - under causal
  attention the padding never influences the positions before it. Every TP
  rank must call it with the same inputs and generator state; pipeline
  stages are not supported.

The CLI loads a sharded checkpoint (any layout) into a single-process model.
The reference has no sampling code.
"""

from __future__ import annotations

import argparse
import json
import os
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..models.gpt import GPT, GPTConfig
from ..parallel.comm import all_gather_dim
from ..parallel.topology import SINGLE


class KVCache:
    """Keys and values of every layer for the tokens seen so far, in
    preallocated ``[B, H, block_size, D]`` buffers, and the decoding step of
    a :class:`GPT` over them (PyTorch ops on the model's parameters). Under
    tensor parallelism each rank caches its own heads; the row-parallel
    outputs are summed over the group (bias added once, after the sum) and the
    vocabulary-sharded logits gathered, so every rank sees the same logits -
    every rank of the group must make the same calls."""

    def __init__(self, model: GPT, batch: int):
        cfg = model.config
        self.model = model
        self.tp = model.tp
        p = model.wte.weight
        self.H, self.D = cfg.n_head // self.tp.world, cfg.n_embd // cfg.n_head
        shape = (batch, self.H, cfg.block_size, self.D)
        self.k = [torch.empty(shape, dtype=p.dtype, device=p.device) for _ in range(cfg.n_layer)]
        self.v = [torch.empty(shape, dtype=p.dtype, device=p.device) for _ in range(cfg.n_layer)]
        self.len = 0

    @staticmethod
    def _ln(ln, x):
        return F.layer_norm(x, ln.normalized_shape, ln.weight, ln.bias, ln.eps)

    def _row(self, x: torch.Tensor, layer) -> torch.Tensor:
        """Row-parallel linear: local partial product, sum over the group, then the full bias."""
        y = F.linear(x, layer.weight)
        if self.tp.enabled:
            dist.all_reduce(y, group=self.tp.group)
        return y + layer.bias if layer.bias is not None else y

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """Run ``tokens`` [B, t] at positions ``len .. len + t - 1`` (the whole
        window when the cache is empty, else one token), append their keys and
        values, and return the logits [B, vocab] of the last one."""
        m, cfg = self.model, self.model.config
        b, t = tokens.shape
        p0 = self.len
        if p0 + t > cfg.block_size or (p0 > 0 and t != 1):
            raise ValueError("KVCache.forward: a full window first, then one token at a time")
        pos = torch.arange(p0, p0 + t, device=tokens.device)
        x = F.embedding(tokens, m.wte.weight) + F.embedding(pos, m.wpe.weight)[None]
        for i, blk in enumerate(m.blocks):
            a = blk.attn
            qkv = F.linear(self._ln(blk.ln_1, x), a.qkv.weight, a.qkv.bias).view(b, t, self.H, 3, self.D)
            q, k, v = (qkv[:, :, :, j].transpose(1, 2) for j in range(3))
            self.k[i][:, :, p0 : p0 + t] = k
            self.v[i][:, :, p0 : p0 + t] = v
            keys, vals = self.k[i][:, :, : p0 + t], self.v[i][:, :, : p0 + t]
            # the window's first pass is causal; a single new token sees every cached one
            y = F.scaled_dot_product_attention(q, keys, vals, is_causal=p0 == 0 and t > 1)
            y = y.transpose(1, 2).reshape(b, t, self.H * self.D)
            x = x + self._row(y, a.proj)
            h = F.gelu(F.linear(self._ln(blk.ln_2, x), blk.mlp.c_fc.weight, blk.mlp.c_fc.bias), approximate="tanh")
            x = x + self._row(h, blk.mlp.c_proj)
        self.len = p0 + t
        x = self._ln(m.ln_f, x[:, -1])
        logits = F.linear(x, m.lm_head.weight)  # this rank's vocabulary shard
        if self.tp.enabled:
            logits = all_gather_dim(logits, self.tp, 1)
        return logits[:, : cfg.vocab_size]


def _sample(logits: torch.Tensor, temperature: float, top_k: Optional[int], generator,
            top_p: Optional[float] = None) -> torch.Tensor:
    logits = logits.float()
    if temperature <= 0:
        return logits.argmax(dim=-1, keepdim=True)
    logits = logits / temperature
    if top_k is not None and top_k < logits.shape[-1]:
        kth = torch.topk(logits, top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    probs = torch.softmax(logits, dim=-1)
    if top_p is not None and top_p < 1.0:
        # nucleus: the most probable tokens whose probabilities sum to top_p (at least one)
        sorted_p, order = probs.sort(dim=-1, descending=True)
        drop = sorted_p.cumsum(dim=-1) - sorted_p >= top_p
        sorted_p = sorted_p.masked_fill(drop, 0.0)
        probs = torch.zeros_like(probs).scatter_(-1, order, sorted_p)
        probs = probs / probs.sum(dim=-1, keepdim=True)
    return torch.multinomial(probs.cpu(), 1, generator=generator).to(logits.device)


def _full_context_logits(model: GPT, idx: torch.Tensor, pad_to: int) -> torch.Tensor:
    cfg = model.config
    ctx = idx[:, -cfg.block_size:]
    n = ctx.shape[1]
    padded = min(cfg.block_size, -(-n // pad_to) * pad_to) if pad_to > 1 else n
    if padded > n:
        ctx = torch.cat([ctx, ctx.new_zeros(ctx.shape[0], padded - n)], dim=1)
    logits, _ = model(ctx)
    return logits[:, n - 1, : cfg.vocab_size]


@torch.no_grad()
def generate(model: GPT, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0,
             top_k: Optional[int] = None, generator: Optional[torch.Generator] = None, pad_to: int = 128,
             use_cache: bool = True, top_p: Optional[float] = None) -> torch.Tensor:
    cfg = model.config
    cache = KVCache(model, idx.shape[0]) if use_cache else None
    was_training = model.training
    model.eval()
    try:
        for _ in range(max_new_tokens):
            if cache is None or idx.shape[1] > cfg.block_size:
                logits = _full_context_logits(model, idx, pad_to)  # window slides: positions shift
            elif cache.len == 0:
                logits = cache.forward(idx)
            else:
                logits = cache.forward(idx[:, -1:])
            nxt = _sample(logits, temperature, top_k, generator, top_p)
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
    ap.add_argument("--top-p", type=float, default=None, help="nucleus sampling")
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
    out = generate(model, idx, a.max_new_tokens, a.temperature, a.top_k, g, top_p=a.top_p)[0].tolist()
    print(decode(out) if decode else ",".join(map(str, out)))


if __name__ == "__main__":
    main()
