"""dstraining_b200: a B200-native 3D-parallel GPT trainer.

Layers (bottom up): ``parallel`` (process grid, collectives, pipeline
schedules, data-parallel reduction, NVLink peer memory), ``ops`` (autograd
ops that run hand-written sm_100a kernels on CUDA bf16 and plain PyTorch
elsewhere), ``models`` (GPT and its pipeline stages), ``optim`` (fp32-master
Adam, fused DP reduce + Adam), ``utils`` (data, checkpoints, timing). The
``dst`` package at the repository root re-exports the reference-compatible
API on top of these.
"""

import os

# Load every kernel when the CUDA context is created instead of at its first
# launch. With lazy loading, the first launch of a kernel waits for the device
# to go idle; a rank with an outstanding NCCL send or receive (a kernel
# spinning until the peer takes part), or a fused collective spinning on a
# peer's flag, never goes idle while that peer is stuck in the same way, so
# both ranks would wait forever. Must be set before the context exists.
os.environ.setdefault("CUDA_MODULE_LOADING", "EAGER")

__version__ = "0.1.0"
