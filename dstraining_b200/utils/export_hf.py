"""Export a trained model in the Hugging Face GPT-2 layout, for serving stacks.

    python -m dstraining_b200.utils.export_hf --ckpt ckpt/ --out gpt2-export [--dtype bfloat16]

Writes ``config.json`` and ``model.safetensors`` that
``transformers.GPT2LMHeadModel.from_pretrained(out)`` loads (and the serving
engines that read that format). The architectures are the same - pre-LN
blocks, tanh GELU (``gelu_new``), learned positions, LayerNorm eps 1e-5 -
with these mappings:

* the fused qkv projection is head-major here (output row ``h*3D + j*D + d``
  for head h, j in q/k/v) and q|k|v-major there (``j*C + h*D + d``): rows are
  permuted;
* Hugging Face's ``Conv1D`` stores weights as ``[in, out]``: every linear
  weight is transposed;
* the LM head is not tied to the token embedding (``tie_word_embeddings``
  false) and keeps only the rows of the real vocabulary (the padding to a
  multiple of 128 is dropped).

The reference has no export; its checkpoints do not exist either.
"""

from __future__ import annotations

import argparse
import json
import os
from typing import Dict

import torch

from ..models.gpt import GPT


def hf_config(model: GPT) -> Dict:
    cfg = model.config
    return {
        "architectures": ["GPT2LMHeadModel"],
        "model_type": "gpt2",
        "vocab_size": cfg.vocab_size,
        "n_positions": cfg.block_size,
        "n_ctx": cfg.block_size,
        "n_embd": cfg.n_embd,
        "n_layer": cfg.n_layer,
        "n_head": cfg.n_head,
        "n_inner": 4 * cfg.n_embd,
        "activation_function": "gelu_new",
        "resid_pdrop": 0.0,
        "embd_pdrop": 0.0,
        "attn_pdrop": 0.0,
        "layer_norm_epsilon": 1e-5,
        "scale_attn_weights": True,
        "tie_word_embeddings": False,
    }


def _qkv_rows(n_head: int, head_dim: int) -> torch.Tensor:
    """Index map: Hugging Face row (j, h, d) <- this model's row (h, j, d)."""
    h = torch.arange(n_head).view(1, n_head, 1)
    j = torch.arange(3).view(3, 1, 1)
    d = torch.arange(head_dim).view(1, 1, head_dim)
    return (h * 3 * head_dim + j * head_dim + d).reshape(-1)


def hf_state_dict(model: GPT, dtype: torch.dtype = torch.float32) -> Dict[str, torch.Tensor]:
    """The model's weights under Hugging Face GPT-2 names and layouts
    (single-process model: load a sharded checkpoint with
    :func:`dstraining_b200.utils.generate.load_model` first)."""
    if model.tp.enabled:
        raise ValueError("export a single-process model (load the checkpoint with tp=1)")
    cfg = model.config
    rows = _qkv_rows(cfg.n_head, cfg.n_embd // cfg.n_head)
    out: Dict[str, torch.Tensor] = {}

    def put(name: str, t: torch.Tensor) -> None:
        out[name] = t.detach().to("cpu", dtype).contiguous()

    put("transformer.wte.weight", model.wte.weight)
    put("transformer.wpe.weight", model.wpe.weight)
    for i, blk in enumerate(model.blocks):
        pre = f"transformer.h.{i}."
        put(pre + "ln_1.weight", blk.ln_1.weight)
        put(pre + "ln_1.bias", blk.ln_1.bias)
        put(pre + "attn.c_attn.weight", blk.attn.qkv.weight[rows].t())
        put(pre + "attn.c_attn.bias", blk.attn.qkv.bias[rows])
        put(pre + "attn.c_proj.weight", blk.attn.proj.weight.t())
        put(pre + "attn.c_proj.bias", blk.attn.proj.bias)
        put(pre + "ln_2.weight", blk.ln_2.weight)
        put(pre + "ln_2.bias", blk.ln_2.bias)
        put(pre + "mlp.c_fc.weight", blk.mlp.c_fc.weight.t())
        put(pre + "mlp.c_fc.bias", blk.mlp.c_fc.bias)
        put(pre + "mlp.c_proj.weight", blk.mlp.c_proj.weight.t())
        put(pre + "mlp.c_proj.bias", blk.mlp.c_proj.bias)
    put("transformer.ln_f.weight", model.ln_f.weight)
    put("transformer.ln_f.bias", model.ln_f.bias)
    put("lm_head.weight", model.lm_head.weight[: cfg.vocab_size])
    return out


def export(model: GPT, out_dir: str, dtype: torch.dtype = torch.float32) -> str:
    """Write ``config.json`` + ``model.safetensors`` into ``out_dir``; returns it."""
    from safetensors.torch import save_file

    os.makedirs(out_dir, exist_ok=True)
    conf = hf_config(model)
    conf["torch_dtype"] = str(dtype).replace("torch.", "")
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(conf, f, indent=1)
    save_file(hf_state_dict(model, dtype), os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
    return out_dir


def main(argv=None) -> None:
    from .generate import load_model

    ap = argparse.ArgumentParser(description="export a checkpoint in the Hugging Face GPT-2 layout")
    ap.add_argument("--ckpt", required=True, help="a checkpoint directory, or a root (its latest complete one)")
    ap.add_argument("--out", required=True)
    ap.add_argument("--dtype", default="float32", choices=["float32", "bfloat16", "float16"])
    a = ap.parse_args(argv)
    model = load_model(a.ckpt)
    print(export(model, a.out, getattr(torch, a.dtype)))


if __name__ == "__main__":
    main()
