"""Model definitions."""

from .gpt import GPT, GPTChunks, GPTConfig, GPTStage  # noqa: F401
