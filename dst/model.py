"""GPT model family (see :mod:`dstraining_b200.models.gpt`)."""

from dstraining_b200.models.gpt import (  # noqa: F401
    GPT,
    VOCAB_PAD_MULTIPLE,
    Block,
    CausalSelfAttention,
    GPTChunks,
    GPTConfig,
    GPTStage,
    MLP,
    core_attention,
)
