"""Autograd ops: native sm_100a kernels on CUDA bf16, PyTorch elsewhere."""
