"""Check a training layout before launching it.

    python -m dstraining_b200.utils.plan --tp 2 --pp 2 --dp 2 --sp --bf16 --vp \
        --layers 24 --heads 16 --embd 2048 --block 2048 --vocab 50304 --batch 32 --micro 2

Takes ``train.py``'s flags and reports, without building the model:

* whether the layout is valid (the same divisibility rules the model and the
  schedules enforce: heads and d_ff by tp, layers by pp x chunks,
  micro-batches by pp for interleaving, sequence by tp under SP);
* whether it stays on the fast native paths on CUDA with ``--bf16``: the
  tcgen05 attention kernels take head size 64 or 128 and run on 128-row
  tiles (other sequence lengths are zero-padded up to one); the fused
  NVLink tensor-parallel kernels need sequence shards of a multiple of 128
  tokens and at most 8 TP ranks; the one-kernel NVLink DP optimizer needs at
  most 8 replicas on one machine (otherwise its NCCL form runs);
* parameters per rank (first, middle and last pipeline stage) and the bytes
  of weights, gradients and optimizer state per rank - bf16 weights and
  gradients plus fp32 master and Adam moments, which the fused DP optimizer
  shards over the DP ranks.
"""

from __future__ import annotations

import argparse
import json
import sys
from typing import Dict, List, Optional

from ..models.gpt import padded_vocab


def layer_params(d: int, tp: int) -> int:
    """Parameters of one block on one TP rank: qkv (3d^2 + 3d) and c_fc (4d^2 + 4d)
    split by rows, proj and c_proj (d^2, 4d^2) split by columns with their
    biases (d each) replicated, two LayerNorms (4d) replicated."""
    return (12 * d * d + 7 * d) // tp + 2 * d + 4 * d


def stage_params(args, stage: int, tp: int) -> int:
    d, layers, pp = args.embd, args.layers, args.pp
    n = (layers // pp) * layer_params(d, tp)
    if stage == 0:
        n += args.vocab * d + args.block * d  # wte (real vocabulary), wpe; replicated over TP
    if stage == pp - 1:
        n += 2 * d + padded_vocab(args.vocab) * d // tp  # ln_f, head over the padded vocabulary (no bias)
    return n


def plan(args) -> Dict:
    if getattr(args, "gpt2", False):  # the preset the trainer applies (GPT-2 124M shape)
        args = argparse.Namespace(**{**vars(args), "layers": 12, "heads": 12, "embd": 768, "block": 1024,
                                     "vocab": 50257})
    tp, pp, dp, v = args.tp, args.pp, args.dp, args.chunks
    errors: List[str] = []
    warnings: List[str] = []
    d, heads, seq = args.embd, args.heads, args.block
    if d % heads:
        errors.append(f"embd {d} not divisible by heads {heads}")
    if heads % tp:
        errors.append(f"heads {heads} not divisible by tp {tp}")
    if (4 * d) % tp or d % tp:
        errors.append(f"embd {d} / d_ff {4 * d} not divisible by tp {tp}")
    if args.layers % (pp * v):
        errors.append(f"layers {args.layers} not divisible by pp x chunks = {pp * v}")
    if args.sp and seq % tp:
        errors.append(f"sequence {seq} not divisible by tp {tp} (sequence parallelism)")
    m = 1
    if pp > 1 or v > 1 or getattr(args, "grad_accum", False):
        if args.batch % args.micro:
            errors.append(f"batch {args.batch} not divisible by micro {args.micro}")
        else:
            m = args.batch // args.micro
        if v > 1 and m % pp:
            errors.append(f"interleaving needs micro-batches ({m}) divisible by pp ({pp})")
    head_dim = d // heads if heads else 0
    native = bool(getattr(args, "bf16", False))
    if native:
        if head_dim not in (64, 128):
            warnings.append(f"head size {head_dim}: native attention takes 64 or 128")
        if seq % 128:
            warnings.append(f"sequence {seq} not a multiple of 128: attention zero-pads it to "
                            f"{-(-seq // 128) * 128} (padded rows computed and discarded)")
        if tp > 1:
            if tp > 8:
                warnings.append("more than 8 TP ranks: fused NVLink TP kernels unavailable (NCCL path)")
            elif seq % tp or (seq // tp) % 128:
                warnings.append(f"sequence shard {seq // max(tp, 1)} not a multiple of 128: fused TP kernels "
                                "unavailable (NCCL + GEMM path)")
        if dp > 8:
            warnings.append("more than 8 DP replicas: the DP reduction runs as NCCL reduce-scatter / all-gather "
                            "around the sharded Adam instead of the one-kernel NVLink path")
    per_stage = [stage_params(args, s, tp) for s in range(pp)] if not errors else []
    fused_dp = native and not getattr(args, "naive_dp", False)
    mem = []
    for n in per_stage:
        weights = 2 * n if native else 4 * n
        grads = 2 * n if native else 4 * n
        opt_state = 12 * n / (dp if fused_dp else 1) if native else 8 * n
        mem.append({"params": n, "weights_gb": round(weights / 2**30, 3), "grads_gb": round(grads / 2**30, 3),
                    "optimizer_gb": round(opt_state / 2**30, 3)})
    return {
        "world": tp * pp * dp,
        "layout": {"tp": tp, "pp": pp, "dp": dp, "chunks": v, "sp": bool(args.sp)},
        "micro_batches": m,
        "tokens_per_step": args.batch * seq * dp,
        "valid": not errors,
        "errors": errors,
        "fast_path_warnings": warnings,
        "per_stage": mem,
        "optimizer": (("fused NVLink DP Adam (state sharded over dp)" if dp <= 8 else
                       "NCCL reduce-scatter + Adam sharded over dp + all-gather") if fused_dp else
                      "fp32-master Adam" if native else "torch Adam (fp32)"),
    }


def main(argv: Optional[List[str]] = None) -> None:
    from ..trainer import parse_args

    report = plan(parse_args(argv))
    print(json.dumps(report, indent=1))
    sys.exit(0 if report["valid"] else 1)


if __name__ == "__main__":
    main()
