"""GPT-2 style pre-LN decoder, tensor/sequence/pipeline parallel by construction.

Per block (Megatron layout): fused head-major QKV column-parallel projection,
causal attention on the local heads, row-parallel output projection; MLP is
column-parallel ``c_fc`` (GELU-tanh) then row-parallel ``c_proj`` with
``d_ff = 4 * d_model``. LayerNorms, embeddings and post-reduction biases are
replicated. The LM head is column-parallel over the vocabulary padded to a
multiple of 128 (independent of tp) and is not tied to ``wte``.

Public contract shared with the reference (``dst/model.py``), because
checkpoints, tests and the pipeline code depend on it:

* module/parameter names: ``wte, wpe, blocks.{i}.{ln_1, attn.qkv, attn.proj,
  ln_2, mlp.c_fc, mlp.c_proj}, ln_f, lm_head`` (and ``chunks.{c}.…`` for
  interleaved stages);
* decomposition-invariant init: every component draws from its own CPU
  generator seeded ``seed * 1000003 + component`` with ids wte=0, wpe=1,
  head=2, block i = 10 + i; inside a block the draw order is qkv, proj, c_fc,
  c_proj; std 0.02 and ``0.02 / sqrt(2 L)`` for the residual projections
  (``dst/model.py:72-103,132,173``);
* ``forward(idx | hidden, targets) -> (logits | None, loss | None)``.

Under sequence parallelism the LayerNorm/residual regions hold
``[B, T/tp, C]``; LayerNorm weights and row-parallel biases then get partial
gradients and :meth:`finalize_grads` sums them over the TP group (one
flattened all-reduce for all of them, not one per parameter).

On CUDA bf16 every op below dispatches to the native sm_100a kernels; the
model code is the same for both paths.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from ..ops import native
from ..ops.attention import causal_attention, core_attention  # noqa: F401  (re-exported API)
from ..ops.cross_entropy import vocab_parallel_cross_entropy
from ..ops.embedding import embed_tokens
from ..ops.layernorm import LayerNorm
from ..ops.recompute import recompute
from ..parallel.comm import gather_from_tp_region
from ..parallel.topology import PP_SINGLE, PPContext, TPContext
from ..utils import trace
from .layers import ColumnParallelLinear, RowParallelLinear

VOCAB_PAD_MULTIPLE = 128

COMP_WTE = 0
COMP_WPE = 1
COMP_HEAD = 2
COMP_BLOCK0 = 10


@dataclass
class GPTConfig:
    """Model shape and parallel features (``dst/model.py:81-95``); d_ff is 4·n_embd."""

    vocab_size: int = 50257
    block_size: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    dropout: float = 0.0
    sequence_parallel: bool = False
    recompute_attention: bool = False
    vocab_parallel_loss: bool = False
    # Full activation recompute (not in the reference): each block keeps only
    # its input and re-runs its forward in backward.
    recompute_blocks: bool = False

    def __post_init__(self):
        if self.dropout != 0.0:
            # No RNG discipline across TP ranks / recompute is implemented, as
            # in the reference; refuse instead of training something else.
            raise ValueError("dropout > 0 is not supported")
        if self.n_embd % self.n_head:
            raise ValueError(f"n_embd {self.n_embd} not divisible by n_head {self.n_head}")


def padded_vocab(vocab_size: int) -> int:
    return -(-vocab_size // VOCAB_PAD_MULTIPLE) * VOCAB_PAD_MULTIPLE


def component_generator(seed: int, component: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed * 1000003 + component)


class CausalSelfAttention(nn.Module):
    """Fused head-major qkv (column-parallel), causal attention over the full
    sequence, row-parallel projection (``dst/model.py:122-167``)."""

    def __init__(self, config: GPTConfig, tp: TPContext, generator: torch.Generator):
        super().__init__()
        if config.n_head % tp.world:
            raise ValueError(f"n_head {config.n_head} not divisible by tp {tp.world}")
        self.config = config
        self.tp = tp
        self.n_head_local = config.n_head // tp.world
        self.head_dim = config.n_embd // config.n_head
        mode = "sequence" if config.sequence_parallel else "replicated"
        resid_std = 0.02 / math.sqrt(2 * config.n_layer)
        self.qkv = ColumnParallelLinear(config.n_embd, 3 * config.n_embd, tp, input_mode=mode, generator=generator)
        self.proj = RowParallelLinear(
            config.n_embd, config.n_embd, tp, output_mode=mode, init_std=resid_std, generator=generator
        )

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        qkv = self.qkv(x)  # sequence is full here even under SP
        y = causal_attention(qkv, self.n_head_local, self.head_dim, self.config.recompute_attention)
        return self.proj(y, residual=residual)


class MLP(nn.Module):
    """c_fc (column-parallel) -> tanh GELU -> c_proj (row-parallel) (``dst/model.py:170-189``)."""

    def __init__(self, config: GPTConfig, tp: TPContext, generator: torch.Generator):
        super().__init__()
        mode = "sequence" if config.sequence_parallel else "replicated"
        resid_std = 0.02 / math.sqrt(2 * config.n_layer)
        self.c_fc = ColumnParallelLinear(config.n_embd, 4 * config.n_embd, tp, input_mode=mode, generator=generator)
        self.c_proj = RowParallelLinear(
            4 * config.n_embd, config.n_embd, tp, output_mode=mode, init_std=resid_std, generator=generator
        )

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if native.active(x, self.c_fc.weight):
            from ..ops.linear import mlp

            return mlp(x, self.c_fc, self.c_proj, residual)
        return self.c_proj(self.c_fc(x, activation="gelu_tanh"), residual=residual)


class Block(nn.Module):
    """Pre-LN block: x + attn(ln_1(x)), then x + mlp(ln_2(x)) (``dst/model.py:192-203``)."""

    def __init__(self, config: GPTConfig, tp: TPContext, generator: torch.Generator):
        super().__init__()
        self.ln_1 = LayerNorm(config.n_embd)
        self.attn = CausalSelfAttention(config, tp, generator)
        self.ln_2 = LayerNorm(config.n_embd)
        self.mlp = MLP(config, tp, generator)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # The residual adds are folded into the row-parallel projections (their
        # GEMM epilogue on the native path).
        x = self.attn(self.ln_1(x), residual=x)
        return self.mlp(self.ln_2(x), residual=x)


def _make_embeddings(config: GPTConfig, seed: int) -> Tuple[nn.Embedding, nn.Embedding]:
    wte = nn.Embedding(config.vocab_size, config.n_embd)
    wpe = nn.Embedding(config.block_size, config.n_embd)
    with torch.no_grad():
        wte.weight.normal_(0.0, 0.02, generator=component_generator(seed, COMP_WTE))
        wpe.weight.normal_(0.0, 0.02, generator=component_generator(seed, COMP_WPE))
    return wte, wpe


def _make_head(config: GPTConfig, tp: TPContext, seed: int) -> ColumnParallelLinear:
    return ColumnParallelLinear(
        config.n_embd,
        padded_vocab(config.vocab_size),
        tp,
        bias=False,
        gather_output=not config.vocab_parallel_loss,
        input_mode="sequence" if config.sequence_parallel else "replicated",
        generator=component_generator(seed, COMP_HEAD),
    )


def _tag_sequence_parallel_replicated(module: nn.Module) -> None:
    for m in module.modules():
        if isinstance(m, nn.LayerNorm):
            for p in m.parameters():
                p.sequence_parallel_replicated = True


def _finalize_grads(module: nn.Module, config: GPTConfig, tp: TPContext) -> None:
    """Sum the partial grads of SP-replicated params over the TP group, as one
    flattened all-reduce (the reference issues one per parameter,
    ``dst/model.py:249-254``)."""
    if not (config.sequence_parallel and tp.enabled):
        return
    grads = [
        p.grad
        for p in module.parameters()
        if getattr(p, "sequence_parallel_replicated", False) and p.grad is not None
    ]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=tp.group)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off : off + n].view_as(g))
        off += n


def _head_loss(config: GPTConfig, tp: TPContext, head: ColumnParallelLinear, x, targets):
    """ln_f output -> (logits | None, loss | None)."""
    if targets is not None and config.vocab_parallel_loss and native.active(x, head.weight):
        # Fused LM head: GEMM tiles reduced to per-row softmax stats on chip.
        from ..ops.fused_head import fused_head_loss

        return None, fused_head_loss(x, head.weight, targets, tp, config.vocab_size, config.sequence_parallel)
    out = head(x)
    if config.vocab_parallel_loss:
        if targets is not None:
            return None, vocab_parallel_cross_entropy(out, targets, tp, config.vocab_size)
        return gather_from_tp_region(out, tp)[..., : config.vocab_size], None
    logits = out[..., : config.vocab_size]
    loss = None
    if targets is not None:
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))
    return logits, loss


class _StageBody(nn.Module):
    """Shared forward for GPT and GPTStage."""

    def _embed(self, idx: torch.Tensor) -> torch.Tensor:
        return embed_tokens(idx, self.wte.weight, self.wpe.weight, self.tp, self.config.sequence_parallel)

    def _run_blocks(self, x: torch.Tensor) -> torch.Tensor:
        full = self.config.recompute_blocks and torch.is_grad_enabled()
        if not trace.enabled() and not full:
            for block in self.blocks:
                x = block(x)
            return x
        for i, block in enumerate(self.blocks):
            with trace.nvtx_range(f"block{i}"):
                x = recompute(block, x) if full else block(x)
        return x

    def finalize_grads(self) -> None:
        """Sum SP-partial grads over TP. Call after backward, before the
        optimizer step; a no-op without sequence parallelism."""
        _finalize_grads(self, self.config, self.tp)


class GPT(_StageBody):
    """The whole model on one TP group."""

    def __init__(self, config: GPTConfig, tp: TPContext, seed: int = 0):
        super().__init__()
        self.config = config
        self.tp = tp
        self.padded_vocab = padded_vocab(config.vocab_size)
        self.wte, self.wpe = _make_embeddings(config, seed)
        self.blocks = nn.ModuleList(
            Block(config, tp, component_generator(seed, COMP_BLOCK0 + i)) for i in range(config.n_layer)
        )
        self.ln_f = LayerNorm(config.n_embd)
        self.lm_head = _make_head(config, tp, seed)
        if config.sequence_parallel:
            _tag_sequence_parallel_replicated(self)

    def ref_param_name(self, name: str) -> str:
        return name

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None):
        x = self._run_blocks(self._embed(idx))
        return _head_loss(self.config, self.tp, self.lm_head, self.ln_f(x), targets)


class GPTStage(_StageBody):
    """One pipeline stage: a contiguous slice of blocks, with the embeddings
    on the first stage and ln_f + head + loss on the last. The interleaved
    schedule passes an explicit ``layer_range`` and virtual first/last flags
    (see :class:`GPTChunks`)."""

    def __init__(
        self,
        config: GPTConfig,
        tp: TPContext,
        pp: PPContext = PP_SINGLE,
        seed: int = 0,
        *,
        layer_range=None,
        is_first: Optional[bool] = None,
        is_last: Optional[bool] = None,
    ):
        super().__init__()
        self.config = config
        self.tp = tp
        self.pp = pp
        self.padded_vocab = padded_vocab(config.vocab_size)
        if layer_range is None:
            if config.n_layer % pp.world:
                raise ValueError(f"n_layer {config.n_layer} not divisible by pp {pp.world}")
            per = config.n_layer // pp.world
            layer_range = (pp.rank * per, (pp.rank + 1) * per)
            is_first, is_last = pp.is_first, pp.is_last
        self.first_layer, self.last_layer = layer_range
        self.is_first_stage = bool(is_first)
        self.is_last_stage = bool(is_last)
        if self.is_first_stage:
            self.wte, self.wpe = _make_embeddings(config, seed)
        self.blocks = nn.ModuleList(
            Block(config, tp, component_generator(seed, COMP_BLOCK0 + layer))
            for layer in range(self.first_layer, self.last_layer)
        )
        if self.is_last_stage:
            self.ln_f = LayerNorm(config.n_embd)
            self.lm_head = _make_head(config, tp, seed)
        if config.sequence_parallel:
            _tag_sequence_parallel_replicated(self)

    def ref_param_name(self, name: str) -> str:
        """Stage-local parameter name -> the full model's name."""
        if name.startswith("blocks."):
            _, idx, rest = name.split(".", 2)
            return f"blocks.{self.first_layer + int(idx)}.{rest}"
        return name

    def forward(self, x: torch.Tensor, targets: Optional[torch.Tensor] = None):
        if self.is_first_stage:
            x = self._embed(x)
        x = self._run_blocks(x)
        if not self.is_last_stage:
            return x
        return _head_loss(self.config, self.tp, self.lm_head, self.ln_f(x), targets)


class GPTChunks(nn.Module):
    """The ``v`` model chunks one rank holds under the interleaved schedule.

    Virtual stage ``k = c * p + r`` is chunk ``c`` of rank ``r`` and holds
    layers ``[k * L/(p v), (k + 1) * L/(p v))``; embeddings live in chunk 0 of
    rank 0, head and loss in chunk ``v-1`` of rank ``p-1``
    (``dst/model.py:381-421``)."""

    def __init__(self, config: GPTConfig, tp: TPContext, pp: PPContext, v: int, seed: int = 0):
        super().__init__()
        p = pp.world
        if config.n_layer % (p * v):
            raise ValueError(f"n_layer {config.n_layer} not divisible by p*v {p * v}")
        per = config.n_layer // (p * v)
        self.config, self.tp, self.pp, self.v = config, tp, pp, v
        self.chunks = nn.ModuleList(
            GPTStage(
                config,
                tp,
                pp,
                seed,
                layer_range=((c * p + pp.rank) * per, (c * p + pp.rank + 1) * per),
                is_first=(pp.rank == 0 and c == 0),
                is_last=(pp.rank == p - 1 and c == v - 1),
            )
            for c in range(v)
        )

    def finalize_grads(self) -> None:
        _finalize_grads(self, self.config, self.tp)

    def ref_param_name(self, name: str) -> str:
        _, c, rest = name.split(".", 2)
        return self.chunks[int(c)].ref_param_name(rest)
