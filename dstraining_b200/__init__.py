"""dstraining_b200: a B200-native 3D-parallel GPT trainer.

Layers (bottom up): ``parallel`` (process grid, collectives, pipeline
schedules, data-parallel reduction, NVLink peer memory), ``ops`` (autograd
ops that run hand-written sm_100a kernels on CUDA bf16 and plain PyTorch
elsewhere), ``models`` (GPT and its pipeline stages), ``optim`` (fp32-master
Adam, fused DP reduce + Adam), ``utils`` (data, checkpoints, timing). The
``dst`` package at the repository root re-exports the reference-compatible
API on top of these.
"""

__version__ = "0.1.0"
