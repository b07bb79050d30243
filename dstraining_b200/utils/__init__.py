"""Data, checkpoints, timing."""
