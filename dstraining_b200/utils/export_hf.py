"""Export a trained model in the Hugging Face GPT-2 layout, for serving stacks,
and import GPT-2 weights in that layout, for fine-tuning.

    python -m dstraining_b200.utils.export_hf --ckpt ckpt/ --out gpt2-export [--dtype bfloat16]
    python -m dstraining_b200.utils.export_hf --import-hf gpt2-dir --ckpt ckpt/
        # then: train.py --ckpt-dir ckpt/ --resume ... (any layout; resharded on load)

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
from ..parallel.topology import SINGLE


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


def import_hf(hf_dir: str, seed: int = 0) -> GPT:
    """A single-process :class:`GPT` (fp32) holding the weights of a Hugging
    Face GPT-2 directory (``config.json`` + ``model.safetensors``; an untied
    or tied head). The inverse of :func:`export`; the padded head rows are
    zero."""
    from safetensors.torch import load_file

    from ..models.gpt import GPTConfig

    with open(os.path.join(hf_dir, "config.json")) as f:
        conf = json.load(f)
    if conf.get("activation_function", "gelu_new") not in ("gelu_new", "gelu_pytorch_tanh"):
        raise ValueError(f"activation {conf.get('activation_function')!r}: this model uses tanh GELU")
    if conf.get("n_inner") not in (None, 4 * conf["n_embd"]):
        raise ValueError("n_inner must be 4 * n_embd")
    cfg = GPTConfig(vocab_size=conf["vocab_size"], block_size=conf["n_positions"], n_layer=conf["n_layer"],
                    n_head=conf["n_head"], n_embd=conf["n_embd"])
    sd = load_file(os.path.join(hf_dir, "model.safetensors"))
    sd = {k if k.startswith(("transformer.", "lm_head.")) else "transformer." + k: v for k, v in sd.items()}
    model = GPT(cfg, SINGLE, seed=seed)
    rows = _qkv_rows(cfg.n_head, cfg.n_embd // cfg.n_head)
    inv = torch.empty_like(rows)
    inv[rows] = torch.arange(rows.numel())

    def get(name: str) -> torch.Tensor:
        return sd[name].float()

    with torch.no_grad():
        model.wte.weight.copy_(get("transformer.wte.weight"))
        model.wpe.weight.copy_(get("transformer.wpe.weight"))
        for i, blk in enumerate(model.blocks):
            pre = f"transformer.h.{i}."
            blk.ln_1.weight.copy_(get(pre + "ln_1.weight"))
            blk.ln_1.bias.copy_(get(pre + "ln_1.bias"))
            blk.attn.qkv.weight.copy_(get(pre + "attn.c_attn.weight").t()[inv])
            blk.attn.qkv.bias.copy_(get(pre + "attn.c_attn.bias")[inv])
            blk.attn.proj.weight.copy_(get(pre + "attn.c_proj.weight").t())
            blk.attn.proj.bias.copy_(get(pre + "attn.c_proj.bias"))
            blk.ln_2.weight.copy_(get(pre + "ln_2.weight"))
            blk.ln_2.bias.copy_(get(pre + "ln_2.bias"))
            blk.mlp.c_fc.weight.copy_(get(pre + "mlp.c_fc.weight").t())
            blk.mlp.c_fc.bias.copy_(get(pre + "mlp.c_fc.bias"))
            blk.mlp.c_proj.weight.copy_(get(pre + "mlp.c_proj.weight").t())
            blk.mlp.c_proj.bias.copy_(get(pre + "mlp.c_proj.bias"))
        model.ln_f.weight.copy_(get("transformer.ln_f.weight"))
        model.ln_f.bias.copy_(get("transformer.ln_f.bias"))
        head = sd.get("lm_head.weight", sd["transformer.wte.weight"]).float()  # tied checkpoints have no head
        model.lm_head.weight.zero_()
        model.lm_head.weight[: cfg.vocab_size].copy_(head)
    return model


def main(argv=None) -> None:
    from . import checkpoint
    from .generate import load_model
    from ..parallel.topology import PP_SINGLE

    ap = argparse.ArgumentParser(description="export to / import from the Hugging Face GPT-2 layout")
    ap.add_argument("--ckpt", required=True,
                    help="export: a checkpoint directory or root; import: the root to write a step-0 checkpoint to")
    ap.add_argument("--out", default=None, help="export: the output directory")
    ap.add_argument("--import-hf", default=None, help="import: a Hugging Face GPT-2 directory")
    ap.add_argument("--dtype", default="float32", choices=["float32", "bfloat16", "float16"])
    a = ap.parse_args(argv)
    if a.import_hf:
        model = import_hf(a.import_hf)
        print(checkpoint.save(a.ckpt, 0, model, None, SINGLE, PP_SINGLE, SINGLE, model.config, 0))
        return
    if not a.out:
        ap.error("--out is required for an export")
    model = load_model(a.ckpt)
    print(export(model, a.out, getattr(torch, a.dtype)))


if __name__ == "__main__":
    main()
